// Launchers of the row-wise kernels (rows.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace ksw {

struct GatherArgs {
  const void* src;              // [src_rows, H]
  int src_dtype;                // F32 / F16 / BF16
  int64_t src_rows;
  int64_t H;
  int top_k;                    // source row of operand row m = sorted[m] / top_k;
                                // 0: source row m itself (valid rows only)
  const int32_t* sorted;        // [max_rows]; NULL: row m reads source row m (quant only)
  const int32_t* num_post_pad;  // rows to process (device)
  int64_t max_rows;
  int64_t numel;                // sentinel of padding slots
  int quant;                    // moe_quant_t
  void* dst;                    // [max_rows, H] dst_dtype / e4m3 / int8
  int dst_dtype;                // for QUANT_NONE: F16 or BF16
  float* scale;                 // FP8: [max_rows, ceil(H/128)], INT8: [max_rows],
                                // FP8_UE8M0: the rows' scale-factor image (bytes)
  // Optional, for top_k in [1, 32] and quant NONE / FP8_BLOCK / FP8_UE8M0:
  // the align's slot map (inv[t * top_k + j] = operand row, -1 = dropped),
  // which switches to the token-major kernel (each source row read and
  // converted once); src_count (device, optional) bounds the source rows.
  const int32_t* inv;
  const int32_t* src_count;
};

struct SumArgs {
  const void* part;             // [splits, T*top_k, H] in part_dtype
  int part_dtype;               // F32, or the output dtype
  int splits;
  int64_t T;
  int top_k;
  int64_t H;
  const void* ids;              // [T*top_k] or NULL (all rows valid)
  int ids_dtype;
  int E;
  void* out;                    // [T, H]
  int out_dtype;
  const int32_t* count_dev;     // optional: only rows t < *count_dev are written
};

struct CombineArgs {
  const void* rows;             // [R, H] rows computed for the flat slots
  int rows_dtype;
  const int32_t* inv;           // [T*top_k] row of each flat slot, -1 = none
  const void* weights;          // [T*top_k]
  int weights_dtype;
  int64_t T;
  int top_k;
  int64_t H;
  void* out;                    // [T, H]
  int out_dtype;
};

int gather_launch(const GatherArgs& a, cudaStream_t s);
int combine_launch(const CombineArgs& a, cudaStream_t s);
int swiglu_reduce_launch(const float* part, int splits, int64_t numel, int64_t I,
                         const int32_t* sorted, const int32_t* num_post_pad, int64_t max_rows,
                         void* act, int act_dtype, cudaStream_t s);
int sum_topk_launch(const SumArgs& a, cudaStream_t s);

}  // namespace ksw
