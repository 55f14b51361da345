/*
 * TEST INFRASTRUCTURE ONLY — the CPU checker for the paged-KV hot path.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load
 * the built oracle/libfe_oracle.so; the product library never links it.
 *
 * A plain-C restatement of the reference's paged-KV operators
 * (Cambridgebit/FlashEngine.cpp):
 *
 *  - append:      src/cuda_kernels.cu:24 (store_kernel) — rows whose slot is
 *                 negative are skipped; with `redirect_negative` set it
 *                 follows the ATen variant src/portable_gpu_ops.cpp:54
 *                 instead, which writes such rows into slot cache_slots-1.
 *  - copy_blocks: no reference implementation exists (the reference never
 *                 copies KV pages); defined as a memcpy of the first `ntok`
 *                 token rows of page `src` onto page `dst`, per layer, K and V.
 *  - gather:      the index_select of src/portable_gpu_ops.cpp:40 made
 *                 ragged: token t of sequence b lives in slot
 *                 pages[kv[b] + t/page]*page + t%page (portable_gpu_ops.cpp:30).
 *  - attention:   src/portable_gpu_ops.cpp:27-44 — per sequence, per query
 *                 head h reading KV head h/(hq/hkv) (repeat_interleave),
 *                 logits = q.k / sqrt(dim), masked to the causal
 *                 (bottom-right: t <= length - qrows + row) or full
 *                 (t < length) pattern of :31, softmax, times V, rounded to
 *                 fp16/bf16 with round-to-nearest-even. The reference does
 *                 the arithmetic in float32 (at::bmm / at::softmax); this
 *                 restatement accumulates in float64 and rounds once, so its
 *                 float32 output is the correctly rounded value of the same
 *                 mathematical expression (the two differ by < 1e-5).
 *
 * Element storage is raw 16-bit patterns (uint16_t); `dtype` 0 = fp16,
 * 1 = bf16.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ---- 16-bit float conversions (IEEE 754 binary16 / bfloat16) ---------- */

static float bits_to_float(uint32_t b) {
  float f;
  memcpy(&f, &b, 4);
  return f;
}
static uint32_t float_to_bits(float f) {
  uint32_t b;
  memcpy(&b, &f, 4);
  return b;
}

float fe_oracle_half_to_float(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t man = h & 0x3ffu;
  if (exp == 0x1f) return bits_to_float(sign | 0x7f800000u | (man << 13));
  if (exp == 0) {
    /* zero or subnormal: value = man * 2^-24 */
    float v = (float)man * 5.9604644775390625e-08f;
    return sign ? -v : v;
  }
  return bits_to_float(sign | ((exp + 112u) << 23) | (man << 13));
}

/* Round-to-nearest-even float -> binary16, with overflow to inf and
 * gradual underflow. */
uint16_t fe_oracle_float_to_half(float f) {
  uint32_t x = float_to_bits(f);
  uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
  uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) /* inf or nan */
    return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
  if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* >= 65520 rounds to inf */
  if (ax < 0x38800000u) {
    /* below the smallest normal 2^-14: subnormal result = round(|f| * 2^24) */
    if (ax < 0x33000000u) return sign; /* < 2^-25 rounds to zero */
    uint32_t e = ax >> 23;
    uint32_t m = (ax & 0x7fffffu) | 0x800000u;
    uint32_t shift = 126u - e; /* 14..24 */
    uint32_t q = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1u);
    if (rem > half || (rem == half && (q & 1u))) q++;
    return (uint16_t)(sign | q);
  }
  uint32_t e = (ax >> 23) - 112u;
  uint32_t m = ax & 0x7fffffu;
  uint32_t q = (e << 10) | (m >> 13);
  uint32_t rem = m & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
  return (uint16_t)(sign | q);
}

float fe_oracle_bf16_to_float(uint16_t h) { return bits_to_float((uint32_t)h << 16); }

uint16_t fe_oracle_float_to_bf16(float f) {
  uint32_t x = float_to_bits(f);
  if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40u); /* quiet nan */
  uint32_t lsb = (x >> 16) & 1u;
  x += 0x7fffu + lsb;
  return (uint16_t)(x >> 16);
}

static float to_float(uint16_t h, int dtype) {
  return dtype ? fe_oracle_bf16_to_float(h) : fe_oracle_half_to_float(h);
}
static uint16_t from_float(float f, int dtype) {
  return dtype ? fe_oracle_float_to_bf16(f) : fe_oracle_float_to_half(f);
}

/* ---- append (store) ---------------------------------------------------- */

void fe_oracle_append(const uint16_t* k, const uint16_t* v, uint16_t* kc, uint16_t* vc,
                      const int64_t* slots, int rows, int width, int cache_slots,
                      int redirect_negative) {
  for (int r = 0; r < rows; ++r) {
    int64_t slot = slots[r];
    if (slot < 0) {
      if (!redirect_negative) continue;
      slot = cache_slots - 1;
    }
    memcpy(kc + slot * (int64_t)width, k + (int64_t)r * width, (size_t)width * 2);
    memcpy(vc + slot * (int64_t)width, v + (int64_t)r * width, (size_t)width * 2);
  }
}

/* ---- rotary embedding -------------------------------------------------- */

/* Restates src/cuda_kernels.cu:19-23 (rope_kernel): q [rows, hq, dim] and
 * k [rows, hkv, dim] rotated in place; with half = rot/2, for each head and
 * j < half, c = cache[pos*rot + j] and s = cache[pos*rot + half + j],
 * x[j] = a*c - b*s, x[j + half] = b*c + a*s, every product and sum rounded
 * to float separately (this file is compiled with -ffp-contract=off), the
 * result rounded to the 16-bit type; dims >= rot are left as they are (rot =
 * dim for the reference's rope, rot < dim for the partial rotary of
 * src/hybrid_model.cpp:44). Rows whose position is outside
 * [0, max_positions) are left unchanged (the product skips them too). */
void fe_oracle_rope(uint16_t* q, uint16_t* k, const int64_t* pos, const float* cache, int rows,
                    int hq, int hkv, int dim, int rot, int max_positions, int dtype) {
  const int half = rot / 2;
  for (int row = 0; row < rows; ++row) {
    if (pos[row] < 0 || pos[row] >= max_positions) continue;
    const float* cs = cache + pos[row] * rot;
    for (int head = 0; head < hq + hkv; ++head) {
      uint16_t* base = head < hq ? q + ((int64_t)row * hq + head) * dim
                                 : k + ((int64_t)row * hkv + (head - hq)) * dim;
      for (int j = 0; j < half; ++j) {
        const float a = to_float(base[j], dtype), b = to_float(base[j + half], dtype);
        const float c = cs[j], s = cs[j + half];
        const float ac = a * c, bs = b * s, bc = b * c, as = a * s;
        const float lo = ac - bs, hi = bc + as;
        base[j] = from_float(lo, dtype);
        base[j + half] = from_float(hi, dtype);
      }
    }
  }
}

/* ---- block copy / copy-on-write ---------------------------------------- */

void fe_oracle_copy_blocks(uint16_t* const* k_pools, uint16_t* const* v_pools, int num_layers,
                           const int32_t* src, const int32_t* dst, const int32_t* ntok,
                           int num_copies, int page, int width) {
  for (int l = 0; l < num_layers; ++l)
    for (int c = 0; c < num_copies; ++c) {
      size_t bytes = (size_t)ntok[c] * width * 2;
      int64_t s = (int64_t)src[c] * page * width, d = (int64_t)dst[c] * page * width;
      memmove(k_pools[l] + d, k_pools[l] + s, bytes);
      memmove(v_pools[l] + d, v_pools[l] + s, bytes);
    }
}

/* ---- gather ------------------------------------------------------------ */

static int64_t seq_length(const int32_t* kv, const int32_t* last, int b, int page) {
  return (int64_t)(kv[b + 1] - kv[b] - 1) * page + last[b];
}

/* out: [sum_b length_b, width], sequences back to back. */
void fe_oracle_gather(const uint16_t* pool, uint16_t* out, const int32_t* kv, const int32_t* pages,
                      const int32_t* last, int batch, int page, int width) {
  int64_t row = 0;
  for (int b = 0; b < batch; ++b) {
    int64_t len = seq_length(kv, last, b, page);
    for (int64_t t = 0; t < len; ++t, ++row) {
      int64_t slot = (int64_t)pages[kv[b] + t / page] * page + t % page;
      memcpy(out + row * width, pool + slot * width, (size_t)width * 2);
    }
  }
}

/* ---- attention --------------------------------------------------------- */

/* q, out: [rows, hq, dim]; pools: [cache_slots, hkv, dim].
 * out_f32 (optional, may be NULL): the float32 result before rounding. */
int fe_oracle_attention(const uint16_t* q, const uint16_t* kpool, const uint16_t* vpool,
                        uint16_t* out, float* out_f32, const int32_t* qo, const int32_t* kv,
                        const int32_t* pages, const int32_t* last, int batch, int hq, int hkv,
                        int dim, int page, int causal, int dtype) {
  int group = hq / hkv;
  double scale = 1.0 / sqrt((double)dim);
  int64_t max_len = 0;
  for (int b = 0; b < batch; ++b) {
    int64_t len = seq_length(kv, last, b, page);
    if (len > max_len) max_len = len;
  }
  double* logits = (double*)malloc(sizeof(double) * (size_t)(max_len > 0 ? max_len : 1));
  int64_t* slot_of = (int64_t*)malloc(sizeof(int64_t) * (size_t)(max_len > 0 ? max_len : 1));
  float* kf = (float*)malloc(sizeof(float) * (size_t)(max_len > 0 ? max_len : 1) * dim);
  float* vf = (float*)malloc(sizeof(float) * (size_t)(max_len > 0 ? max_len : 1) * dim);
  double* acc = (double*)malloc(sizeof(double) * (size_t)dim);
  float* qf = (float*)malloc(sizeof(float) * (size_t)dim);
  if (!logits || !slot_of || !kf || !vf || !acc || !qf) {
    free(logits); free(slot_of); free(kf); free(vf); free(acc); free(qf);
    return 1;
  }
  for (int b = 0; b < batch; ++b) {
    int64_t len = seq_length(kv, last, b, page);
    int qrows = qo[b + 1] - qo[b];
    if (qrows <= 0) continue;
    for (int64_t t = 0; t < len; ++t)
      slot_of[t] = (int64_t)pages[kv[b] + t / page] * page + t % page;
    for (int kh = 0; kh < hkv; ++kh) {
      for (int64_t t = 0; t < len; ++t)
        for (int d = 0; d < dim; ++d) {
          int64_t off = (slot_of[t] * hkv + kh) * dim + d;
          kf[t * dim + d] = to_float(kpool[off], dtype);
          vf[t * dim + d] = to_float(vpool[off], dtype);
        }
      for (int r = qo[b]; r < qo[b + 1]; ++r) {
        int64_t visible = causal ? len - qrows + (r - qo[b]) + 1 : len;
        if (visible > len) visible = len;
        for (int g = 0; g < group; ++g) {
          int h = kh * group + g;
          const uint16_t* qrow = q + ((int64_t)r * hq + h) * dim;
          for (int d = 0; d < dim; ++d) qf[d] = to_float(qrow[d], dtype);
          double mx = -INFINITY;
          for (int64_t t = 0; t < visible; ++t) {
            double s = 0.0;
            const float* kr = kf + t * dim;
            for (int d = 0; d < dim; ++d) s += (double)qf[d] * (double)kr[d];
            s *= scale;
            logits[t] = s;
            if (s > mx) mx = s;
          }
          double sum = 0.0;
          for (int64_t t = 0; t < visible; ++t) {
            logits[t] = exp(logits[t] - mx);
            sum += logits[t];
          }
          for (int d = 0; d < dim; ++d) acc[d] = 0.0;
          for (int64_t t = 0; t < visible; ++t) {
            double p = logits[t] / sum;
            const float* vr = vf + t * dim;
            for (int d = 0; d < dim; ++d) acc[d] += p * (double)vr[d];
          }
          uint16_t* orow = out + ((int64_t)r * hq + h) * dim;
          for (int d = 0; d < dim; ++d) {
            float o = visible > 0 ? (float)acc[d] : NAN;
            orow[d] = from_float(o, dtype);
            if (out_f32) out_f32[((int64_t)r * hq + h) * dim + d] = o;
          }
        }
      }
    }
  }
  free(logits); free(slot_of); free(kf); free(vf); free(acc); free(qf);
  return 0;
}
