// Device-side step metadata and work lists: the arguments of the planning
// kernel (fe_plan_device.cu) that fe_attn_plan_prepare_device and
// fe_step_prepare_device (fe_attn.cu) launch.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace fe {

struct DevPlanArgs {
  int mode;  // 0: the caller's qo/kv/pages/last; 1: build them from block tables
  // mode 1 inputs (device): block_tables[b * stride + i] is page i of sequence
  // b; starts[b] its first position written this step (< 0: padding entry)
  const int32_t* tables;
  int64_t stride;
  const int32_t* starts;
  int rows_per_seq;
  int64_t* slots;      // mode 1 output: [batch * rows_per_seq], -1 for padding rows
  int64_t* positions;  // mode 1 output: [batch * rows_per_seq]
  // mode 0 inputs (device), the layout of fe_attn_plan_prepare
  const int32_t* qo;
  const int32_t* kv;
  const int32_t* pages;
  const int32_t* last;
  int batch, rows;
  // plan configuration and capacities
  int hq, hkv, dim, page, max_batch, max_pages, num_blocks, dec_heads, grid_cap, dec_grid_cap;
  int max_items, max_groups;
  int64_t partial_capacity, meta_cap;
  // outputs: the packed work lists (fe_attn_plan.h layout), split counters
  uint8_t* meta;
  int32_t* counters;
  unsigned int* err;
  // scratch (device): per-sequence arrays
  int32_t* s_qo;    // [max_batch + 1]
  int32_t* s_kv;    // [max_batch + 1]
  int32_t* s_last;  // [max_batch]
  int32_t* s_cnt;   // [3 * (max_batch + 1)]: row-unit, decode-item and group offsets
  int64_t* s_pref;  // [2 * (max_batch + 1)]: decode-tile and split-record-float offsets
};

// Scratch bytes the kernel needs for a plan of `max_batch` sequences.
size_t plan_device_scratch_bytes(int max_batch);
// Point the scratch arrays of `a` (a.max_batch set) into `base`.
void plan_device_bind_scratch(DevPlanArgs& a, void* base);
// One 1024-thread CTA on `stream`; returns an fe_status.
int plan_device_launch(const DevPlanArgs& a, cudaStream_t stream);

}  // namespace fe
