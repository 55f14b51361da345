/*
 * fe_kv.h — C ABI of the B200 (sm_100a) paged-KV hot path for FlashEngine.cpp.
 *
 * Drop-in for the KV and attention operators behind the reference's CUDA
 * DeviceModel (Cambridgebit/FlashEngine.cpp include/fe/native_cuda.hpp:6-14):
 * K/V append through the slot mapping, paged GQA attention (decode, chunked
 * prefill, speculative verify) over per-sequence block tables, plus a
 * block-copy / copy-on-write operator the reference does not have.
 *
 * Conventions
 *  - Every entry point returns an fe_status; 0 (FE_OK) is success. No C++
 *    exception crosses this boundary. fe_last_error() returns a detail string
 *    for the calling thread's most recent failure.
 *  - `stream` is a cudaStream_t passed as void* (0 = legacy default stream),
 *    the same convention as the reference's `void* stream`.
 *  - Element data are fp16 or bf16 (`dtype`: FE_DTYPE_F16 / FE_DTYPE_BF16).
 *    `bf16` in the shim (fe_native_cuda.hpp) maps to FE_DTYPE_BF16.
 *  - KV pools are laid out as in the reference (src/cuda_model.cpp:60):
 *    [num_blocks + 1, page, hkv, dim], i.e. a flat [cache_slots, hkv*dim]
 *    with cache_slots = (num_blocks + 1) * page. The last page
 *    (index num_blocks) is the graph-padding page and is never handed to a
 *    request.
 *  - Device pointers unless stated "host".
 */
#ifndef FE_KV_H_
#define FE_KV_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FE_KV_ABI_VERSION 1

typedef enum fe_status {
  FE_OK = 0,
  FE_ERR_INVALID_ARGUMENT = 1, /* bad shape, null pointer, unsupported combination */
  FE_ERR_CAPACITY = 2,         /* batch/pages/work beyond the plan's fixed capacity */
  FE_ERR_CONTEXT = 3,          /* a sequence's length < its query rows, or > max context */
  FE_ERR_CUDA = 4,             /* a CUDA runtime call failed (detail in fe_last_error) */
  FE_ERR_UNSUPPORTED = 5,      /* head_dim / page size / group size not compiled */
  FE_ERR_DEVICE = 6,           /* a kernel recorded an error (e.g. out-of-range slot) */
  FE_ERR_NO_DEVICE = 7         /* no usable sm_100 device */
} fe_status;

typedef enum fe_dtype { FE_DTYPE_F16 = 0, FE_DTYPE_BF16 = 1 } fe_dtype;

/* Bits reported by fe_device_errors(). */
#define FE_DEVERR_SLOT_RANGE 0x1u  /* append: slot >= cache_slots (row skipped) */
#define FE_DEVERR_PAGE_RANGE 0x2u  /* copy/clear: page index out of range (copy skipped) */
#define FE_DEVERR_NTOK_RANGE 0x4u  /* copy: ntok outside [0, page] (copy skipped) */
#define FE_DEVERR_TIMEOUT 0x8u     /* attention: a pipeline wait exceeded its bound */
#define FE_DEVERR_SMEM_ALIGN 0x10u /* attention: dynamic shared memory not 1 KiB aligned (launch skipped) */
#define FE_DEVERR_POS_RANGE 0x20u  /* rope: position outside [0, max_positions) (row skipped) */
#define FE_DEVERR_PLAN 0x40u       /* device-side prepare: invalid step or capacity (plan emptied) */

const char* fe_status_string(int status);
const char* fe_last_error(void);
int fe_abi_version(void);

/* Read and clear the device-side error bits of the current device (see
 * FE_DEVERR_*). Synchronises `stream`. */
int fe_device_errors(void* stream, uint32_t* bits_out);

/* ------------------------------------------------------------------------
 * K/V append. Replaces fe::cuda::store (include/fe/native_cuda.hpp:14;
 * src/cuda_kernels.cu:24 store_kernel and :34 its launcher).
 *   k, v:        [rows, width] new post-RoPE keys / values (width = hkv*dim)
 *   k_pool/v_pool: [cache_slots, width]
 *   slots:       int64 [rows] (device); slot < 0 rows are skipped (graph
 *                padding, as the reference CUDA kernel does); a slot
 *                >= cache_slots is skipped and raises FE_DEVERR_SLOT_RANGE.
 * Bit-exact copy. width must be a multiple of 8 elements (16 bytes).
 * ------------------------------------------------------------------------ */
int fe_kv_append(const void* k, const void* v, void* k_pool, void* v_pool, const int64_t* slots,
                 int rows, int width, int dtype, int cache_slots, void* stream);

/* ------------------------------------------------------------------------
 * Block copy / copy-on-write. No reference counterpart: the reference
 * shares only whole published pages and never copies one
 * (src/scheduler.cpp:6-29). For each copy c and each layer l, token rows
 * [0, ntok[c]) of page src[c] are copied onto page dst[c] in both
 * k_pools[l] and v_pools[l] (ntok = page copies a whole block; a smaller
 * ntok is the copy-on-write of a shared partial tail block).
 *   k_pools, v_pools: HOST arrays of num_layers device pool pointers
 *                     (num_layers <= FE_MAX_LAYERS)
 *   src, dst, ntok:   int32 [num_copies] (device)
 * Source and destination pages of one call must not overlap.
 * ------------------------------------------------------------------------ */
#define FE_MAX_LAYERS 128
int fe_kv_copy_blocks(void* const* k_pools, void* const* v_pools, int num_layers,
                      const int32_t* src, const int32_t* dst, const int32_t* ntok, int num_copies,
                      int page, int width, int num_pages_total, int dtype, void* stream);

/* Copy lists for forked sequences (no reference counterpart; HOST memory
 * only, needs no GPU). The reference shares only whole published pages and
 * recomputes the rest of a shared prefix by prefill (src/scheduler.cpp:6-29);
 * a fork that copies KV instead gives, for each fork f, the parent's block
 * table parent_tables[parent_off[f] .. parent_off[f+1]), the child's table
 * child_tables[child_off[f] .. child_off[f+1]) as the scheduler assigned it
 * (the parent's full pages it shares, then pages of its own) and the
 * length fork_len[f] of the prefix the child continues from. For every page
 * j < ceil(fork_len/page) the child does not share, one copy entry
 * (src = parent[j], dst = child[j], ntok = the prefix tokens on that page:
 * page, or fork_len % page for the tail) is written to src/dst/ntok, ready
 * for fe_kv_copy_blocks, which must run before either sequence appends.
 * Rejected with FE_ERR_INVALID_ARGUMENT: a shared page that is not full (both
 * sequences would append into it: the copy-on-write case), a child page that
 * is one of the parent's pages at another position, a fork length beyond
 * either table. FE_ERR_CAPACITY when the copies exceed `capacity`.
 * *num_copies receives the number of entries written. */
int fe_kv_fork_copies(int num_forks, const int32_t* parent_tables, const int32_t* parent_off,
                      const int32_t* child_tables, const int32_t* child_off,
                      const int64_t* fork_len, int page, int32_t* src, int32_t* dst,
                      int32_t* ntok, int capacity, int* num_copies);

/* Zero-fill whole pages (e.g. the graph-padding page num_blocks, which the
 * reference gets from at::zeros at start-up, src/cuda_model.cpp:60).
 *   pools: HOST array of num_pools device pool pointers
 *   pages: int32 [num_pages] (device) */
int fe_kv_clear_pages(void* const* pools, int num_pools, const int32_t* pages, int num_pages,
                      int page, int width, int num_pages_total, int dtype, void* stream);

/* Gather the KV of whole sequences into a dense buffer: the index_select
 * of the reference ATen path (src/portable_gpu_ops.cpp:40) without its
 * padding to max_context. Token t of sequence b is read from slot
 * pages[kv[b] + t/page]*page + t%page, and written to row
 * kv_row_offset[b] + t of `out` ([sum of lengths, width]).
 *   kv, pages, last, kv_row_offset: int32 (device), as in prepare. */
int fe_kv_gather(const void* pool, void* out, const int32_t* kv, const int32_t* pages,
                 const int32_t* last, const int32_t* row_offset, int batch, int max_len, int page,
                 int width, int dtype, void* stream);

/* ------------------------------------------------------------------------
 * Rotary embedding. Replaces fe::cuda::rope (include/fe/native_cuda.hpp:13;
 * src/cuda_kernels.cu:19-23 rope_kernel and :33 its launcher), bit-exact:
 * with r = rotary_dim / 2, for each head and pair (j, j + r), j < r, with
 * c = cache[pos*rotary_dim + j] and s = cache[pos*rotary_dim + r + j] (fp32
 * cache [max_positions, rotary_dim], cos then sin), x[j] = a*c - b*s and
 * x[j + r] = b*c + a*s, each product and sum rounded to fp32 separately, the
 * result rounded to the 16-bit type. rotary_dim = dim is the reference's
 * rope; rotary_dim < dim rotates only the leading dims (the partial rotary of
 * Qwen3.5 full-attention layers, src/hybrid_model.cpp:44) and leaves the rest.
 *   q: [rows, hq, dim], k: [rows, hkv, dim] (rotated in place; hq may be 0)
 *   pos: int64 [rows] (device). A position outside [0, max_positions) leaves
 *        its row unrotated and raises FE_DEVERR_POS_RANGE (the reference
 *        reads out of bounds there).
 * dim and rotary_dim multiples of 4, rotary_dim <= dim; q/k 4-byte aligned,
 * cache 8-byte aligned.
 * ------------------------------------------------------------------------ */
int fe_rope(void* q, void* k, const int64_t* pos, const float* cache, int rows, int hq, int hkv,
            int dim, int rotary_dim, int max_positions, int dtype, void* stream);

/* Fused RoPE + K/V append (one launch): rotates q in place, and writes the
 * rotated keys and the values to the pools through the slot mapping exactly
 * as fe_rope followed by fe_kv_append would (slot < 0 skipped, slot >=
 * cache_slots skipped and flagged). k and v ([rows, hkv, dim]) are read
 * only; when k_out is not NULL the rotated keys are also written there (k_out
 * may equal k). Pools are [cache_slots, hkv*dim]. */
int fe_rope_append(void* q, const void* k, const void* v, void* k_out, void* k_pool,
                   void* v_pool, const int64_t* slots, const int64_t* pos, const float* cache,
                   int rows, int hq, int hkv, int dim, int rotary_dim, int max_positions,
                   int dtype, int64_t cache_slots, void* stream);

/* ------------------------------------------------------------------------
 * Greedy speculative acceptance. Replaces fe::cuda::accept
 * (include/fe/native_cuda.hpp:15; src/cuda_kernels.cu:25 accept_kernel and
 * :35 its launcher). For each row b: m = the number of leading draft tokens
 * draft[b, i] equal to verify[b, i]; out[b, 0..m) = those drafts,
 * out[b, m] = verify[b, m], out[b, k+1] = m + 1; out[b, m+1..k] untouched.
 *   draft: int64 [batch, k], verify: int64 [batch, k+1], out: int64 [batch, k+2]
 * ------------------------------------------------------------------------ */
int fe_accept(const int64_t* draft, const int64_t* verify, int64_t* out, int batch, int k,
              void* stream);

/* ------------------------------------------------------------------------
 * Paged attention plan. Replaces fe::cuda::create_plan / destroy_plan /
 * prepare_plan (include/fe/native_cuda.hpp:7-9; src/flashinfer_attention.cu:22-34).
 * ------------------------------------------------------------------------ */
typedef struct fe_attn_plan fe_attn_plan;

/* head_dim 128 (as src/flashinfer_attention.cu:23 requires) or 256 (the
 * full-attention layers of hybrid and DFlash draft models, which the reference
 * serves through ATen with any head_dim: src/hybrid_model.cpp:98,
 * src/block_draft.cpp:38); page a multiple of 16; hq a multiple of hkv with
 * hq/hkv <= 16.
 * max_pages = per-sequence page capacity (the reference passes
 * ceil(max_model_len/page)+1, src/cuda_model.cpp:118). Allocates the plan's
 * fixed device workspaces on the current device. */
int fe_attn_plan_create(int hq, int hkv, int dim, int page, int max_batch, int max_pages,
                        int dtype, int num_blocks, fe_attn_plan** plan_out);
int fe_attn_plan_destroy(fe_attn_plan* plan);

/* Per-step metadata, HOST pointers (as fe::cuda::prepare_plan):
 *   qo[batch+1]   query-row prefix sums (rows per sequence: 1 = decode,
 *                 k+1 = verify, chunk = prefill)
 *   kv[batch+1]   page-count prefix sums into `pages`
 *   pages[kv[batch]] physical page ids, each in [0, num_blocks]
 *   last[batch]   tokens in each sequence's last page, 1..page
 * length_b = (kv[b+1]-kv[b]-1)*page + last[b] keys; query row r of
 * sequence b is its (r - qo[b])-th of qrows_b = qo[b+1]-qo[b] rows.
 * Builds the work list on the host and uploads it with one async copy on
 * `stream` into fixed device buffers, so a CUDA graph that captured
 * fe_attn_run replays correctly after any later prepare (graph != 0 only
 * asserts that the row count is unchanged). */
int fe_attn_plan_prepare(fe_attn_plan* plan, const int32_t* qo, const int32_t* kv,
                         const int32_t* pages, const int32_t* last, int batch, int rows, int graph,
                         void* stream);

/* Paged GQA attention. Replaces fe::cuda::attention
 * (include/fe/native_cuda.hpp:10; src/flashinfer_attention.cu:35-44).
 *   q, out: [rows, hq, dim]; k_pool, v_pool: [cache_slots, hkv, dim]
 *           (dim = the plan's head_dim, 128 or 256)
 *   causal != 0: row i of a sequence with qrows rows sees keys
 *                t <= length - qrows + i (bottom-right aligned);
 *   causal == 0: every row sees t < length (DFlash draft / block verify).
 * Scale 1/sqrt(dim); fp32 accumulation; output rounded to nearest even.
 * A step prepared outside graph mode that mixes decode rows with multi-row
 * sequences may run its two kernels side by side: the multi-row kernel on a
 * stream the plan owns, forked from `stream` by an event and joined back
 * before the call returns, so the call is ordered on `stream` as usual (and
 * a capture of `stream` records the fork and the join). */
int fe_attn_run(fe_attn_plan* plan, const void* q, const void* k_pool, const void* v_pool,
                void* out, int causal, void* stream);

/* fe_attn_run restricted to some of the prepared work: FE_ATTN_LISTS_DECODE
 * (the rows that run on the decode kernel, and their split-K merge) and/or
 * FE_ATTN_LISTS_ROWS (multi-row sequences on the tcgen05 kernel).
 * fe_attn_run is FE_ATTN_LISTS_ALL. Calling the two parts back to back on one
 * stream does the same work as one fe_attn_run (used to time each kernel). */
#define FE_ATTN_LISTS_DECODE 1
#define FE_ATTN_LISTS_ROWS 2
#define FE_ATTN_LISTS_ALL 3
int fe_attn_run_lists(fe_attn_plan* plan, const void* q, const void* k_pool, const void* v_pool,
                      void* out, int causal, int lists, void* stream);

/* Decode attention that allocates nothing. No counterpart in the reference:
 * it is for callers that cannot call cudaMalloc where they run attention
 * (hosts that give all free device memory to their own pool allocator at
 * start-up, so a later allocation fails; hot loops where an allocation,
 * which may synchronise the device, is not allowed). Same arithmetic as
 * fe_attn_run for one query row per sequence, but no plan: kv, pages and
 * last are DEVICE int32 arrays laid out as in fe_attn_plan_prepare, and the
 * work split is derived on the device.
 * head_dim 128 only: q and out are [batch, hq, 128], row b of q/out belongs
 * to sequence b; pools are [cache_slots, hkv, 128].
 * Split-K scratch is a fixed 16 MiB (+64 KiB counters) array inside the
 * library that every GPU loading it holds until exit; batch x KV-head groups
 * beyond 16384 is rejected with FE_ERR_CAPACITY, and batches whose split
 * records would not fit that array run every sequence unsplit (same
 * results, less parallelism for long contexts). The first call on a device
 * resolves that array's device address and sets kernel attributes — make it
 * before any stream capture. Calls share the array: sequential calls are
 * safe, calls that overlap on the GPU race. Out-of-range page ids or last
 * values are reported through fe_device_errors. */
int fe_paged_decode_noalloc(const void* q, const void* k_pool, const void* v_pool, void* out,
                            const int32_t* kv, const int32_t* pages, const int32_t* last,
                            int batch, int hq, int hkv, int page, int num_blocks, int max_pages,
                            int dtype, void* stream);

/* ------------------------------------------------------------------------
 * Device-side step preparation (no reference counterpart: replaces the host
 * loops of CudaModel::prepare, src/cuda_model.cpp:131-142, and the host
 * planning plus pageable H2D copies of prepare_plan,
 * src/flashinfer_attention.cu:29-34). Every array argument is DEVICE memory
 * and nothing is read back on the host, so both calls can be captured in a
 * CUDA graph together with the append and attention: a decode or verify
 * step then replays with no host work at all.
 *
 * Both leave the plan in graph mode (the attention kernels launch at full
 * width; batch and rows must stay those of the first graph prepare). The
 * work lists are built on the device by one kernel on `stream`: the decode
 * list is the host planner's exact-cut list item for item (identical split
 * points, bit-identical outputs); prefill/verify units (never split) are
 * dealt to the CTAs by cost, longest first, in snake order (at most 8192 such
 * units). Invalid metadata or exceeded capacity does not fail the call (it
 * is not seen on the host): the plan is emptied, attention writes nothing,
 * and FE_DEVERR_PLAN is raised (fe_device_errors).
 * ------------------------------------------------------------------------ */
/* The caller's device metadata, in the layout of fe_attn_plan_prepare. */
int fe_attn_plan_prepare_device(fe_attn_plan* plan, const int32_t* qo, const int32_t* kv,
                                const int32_t* pages, const int32_t* last, int batch, int rows,
                                void* stream);
/* The slot mapping too (CudaModel::prepare): sequence b (b < batch) writes
 * rows_per_seq tokens at positions starts[b] .. starts[b]+rows_per_seq-1
 * through its block-table row block_tables[b*table_stride ...] (int32 page
 * ids, at least ceil((starts[b]+rows_per_seq)/page) of them). starts[b] < 0
 * marks a padding entry of a graph bucket: slot -1 (the append skips it),
 * position j, the dummy page num_blocks, last = rows_per_seq (as
 * src/cuda_model.cpp:138). Writes slots[batch*rows_per_seq] and
 * positions[batch*rows_per_seq] (int64, device) for fe_kv_append / fe_rope*,
 * and plans attention over qo[b] = b*rows_per_seq, the first
 * ceil(length/page) pages of each row, last = (length-1) % page + 1. */
int fe_step_prepare_device(fe_attn_plan* plan, const int32_t* block_tables, int table_stride,
                           const int32_t* starts, int batch, int rows_per_seq, int64_t* slots,
                           int64_t* positions, void* stream);

/* Introspection of the last prepare (host-side numbers, no sync; after a
 * device-side prepare the item counts read -1). */
typedef struct fe_attn_plan_info {
  int batch, rows;
  int decode_items, prefill_items; /* work items queued for the two kernels */
  int split_sequences;             /* (sequence, kv head) pairs split over > 1 item */
  int chunk_tiles;                 /* key tiles (16 tokens) per decode item */
  int grid_ctas;                   /* persistent CTAs launched by fe_attn_run */
  int64_t kv_tokens;               /* sum of sequence lengths */
} fe_attn_plan_info;
int fe_attn_plan_get_info(const fe_attn_plan* plan, fe_attn_plan_info* info);

/* ------------------------------------------------------------------------
 * Test hooks (no reference counterpart): exercise the host planner without
 * a GPU.
 * ------------------------------------------------------------------------ */
/* A plan with no device state; fe_attn_plan_prepare() then only validates
 * and builds the work list, for `grid_cap` persistent CTAs. */
int fe_attn_plan_create_host(int hq, int hkv, int dim, int page, int max_batch, int max_pages,
                             int dtype, int num_blocks, int grid_cap, fe_attn_plan** plan_out);
/* Copy the packed work-list metadata of the last prepare into `dst` (at most
 * `cap` bytes); *bytes receives its full size. Layout: fe_attn_plan.h. */
int fe_attn_plan_debug_meta(const fe_attn_plan* plan, void* dst, int64_t cap, int64_t* bytes);
/* Copy the plan's DEVICE metadata (what the kernels read; at most `cap`
 * bytes) into host memory `dst`; synchronises `stream`. */
int fe_attn_plan_debug_device_meta(const fe_attn_plan* plan, void* dst, int64_t cap, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FE_KV_H_ */
