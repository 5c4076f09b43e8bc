// Internal launchers shared between the translation units of the library.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace ksw {

// ----- align.cu -----
int64_t align_buffer_len(int64_t numel, int E, int BM);
int64_t align_small_max();  // routed rows up to which align is one launch
size_t align_workspace_bytes(int64_t numel, int E);
int align_validate(int64_t numel, int E, int BM);
// valid_dev (optional): only the first *valid_dev * valid_mult flat ids
// take part; the rest are dropped like ids outside [0, E).
// inv (optional, [numel]): receives the slot of every flat id that takes
// part, i.e. inv[sorted[m]] = m, and -1 for ids outside [0, E); entries of
// ids past the valid count are not written.
int align_launch(const void* ids, int ids_dtype, int64_t numel, int E, int BM,
                 int32_t* sorted, int32_t* expert_ids, int32_t* num_post_pad,
                 void* workspace, size_t ws_bytes, cudaStream_t s,
                 const int32_t* valid_dev = nullptr, int valid_mult = 1,
                 int32_t* inv = nullptr);

// ----- gemm.cu -----
// Row-block height of the grouped GEMMs (and the align block size they need).
constexpr int kBlockM = 128;

struct GroupedGemmArgs {
  int quant;                   // moe_quant_t
  int compute_dtype;           // F16 or BF16 for QUANT_NONE
  const void* a;               // [rows, K] operand rows in expert-sorted order
  const float* a_scale;        // FP8: [rows, ceil(K/128)], INT8: [rows]
  const void* b;               // [E, N, K] expert weights
  const float* b_scale;        // FP8: [E, ceil(N/128), ceil(K/128)], INT8: [E, N]
  const int32_t* sorted_ids;   // [rows]
  const int32_t* expert_ids;   // [rows / kBlockM]
  const int32_t* num_post_pad; // [1]
  int64_t rows;                // buffer length (multiple of kBlockM)
  int64_t numel;               // T * k: sorted_ids sentinel
  int num_experts;
  int64_t n;                   // output columns per expert (rows of B)
  int64_t k;                   // reduction length
  // epilogue
  void* out;                   // gate-up: act [rows, n/2]; down: f32 [splits, numel, n]
  const void* row_weights;     // down: [numel] weight of each flat row
  int row_weights_dtype;
  int splits;                  // down: K splits (partial sums summed later)
  int out_dtype;               // down: rows dtype, F32 (0, default) or the 16-bit act dtype
  int32_t* status;
  int block_n;                 // 0 = heuristic
  // 1 when the align outputs (sorted_ids, expert_ids, num_post_pad) were
  // written at least two kernels earlier in the stream, so the GEMM may read
  // them, and request its first weight tiles, before waiting on the kernel
  // that produced its A operand (programmatic dependent launch).
  int early_meta;
};


// ----- decode.cu -----
// Routed rows up to which moe_fused_experts streams the weights through
// two CUDA-core kernels instead of the align/gather/GEMM pipeline (when the
// weights it streams are also small: decode_path_fits).
constexpr int64_t kDecodeMaxRows = 16;

struct DecodeArgs {
  int64_t T, H, I;
  int top_k, E;
  int act_dtype, ids_dtype, weights_dtype;
  const void* hidden;   // [T, H] act dtype
  const void* w13;      // [E, 2I, H] regrouped, act dtype
  const void* w2;       // [E, H, I]
  const void* ids;      // [T, top_k]
  const void* weights;  // [T, top_k]
  void* act;            // [T*top_k, I] scratch
  void* out;            // [T, H]
  // fp32 router logits [T, E] (E <= 256): the gate-up kernel routes the
  // tokens itself and writes ids / weights; null when they are given
  const void* logits = nullptr;
  int renorm = 1;
};

// The decode kernel routes in-kernel for fp32 logits over at most this many experts.
constexpr int kDecodeRouteMaxExperts = 256;

bool decode_path_fits(int64_t T, int top_k, int64_t H, int64_t I, int act_dtype);
bool decode_path_enabled();  // false when MOE_NO_DECODE_PATH=1
// stage 0: gate-up + SiLU*up into act; stage 1: down + weighted top-k sum
int decode_launch(const DecodeArgs& d, int stage, cudaStream_t s);

int gemm_gate_up_launch(const GroupedGemmArgs& a, cudaStream_t s);
int gemm_down_launch(const GroupedGemmArgs& a, cudaStream_t s);
int gemm_gate_up_split_launch(const GroupedGemmArgs& a, cudaStream_t s);

}  // namespace ksw
