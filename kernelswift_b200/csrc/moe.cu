// moe_fused_experts: the whole expert computation of
// kernels/track1-triton/fused_moe/base.py:50-76 as six launches on the
// caller's stream, with no host synchronisation (two weight-streaming
// launches instead when at most 16 rows are routed, csrc/decode.cu):
//
//   1. align      topk_ids -> sorted_token_ids, expert_ids, num_post_pad
//   2. gather     hidden rows in expert-sorted order (+cast / quantise)
//   3. gate-up    grouped tcgen05 GEMM, SiLU(gate)*up fused      [L, I]
//   4. (quant)    per-row quantisation of the activation (W8A8 modes)
//   5. down       grouped tcgen05 GEMM, topk weight fused, optional K split
//   6. sum_topk   out[t] = sum over splits and slots, cast to act dtype
//
// Also exports the stages one by one (moe_gather_rows, moe_gemm_gate_up,
// moe_gemm_down, moe_sum_topk) for callers that build their own pipeline
// (expert parallelism) and for stage-level tests.
#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "internal.h"
#include "rows.h"

namespace ksw {
namespace {

struct Plan {
  int64_t T, H, I, numel, L;
  int E, k;
  int quant;
  int compute_dtype;     // operand dtype for QUANT_NONE
  int a_dtype;           // dtype of the gathered operand
  int act_dtype;         // dtype of the gate-up output (bf16/f16)
  int splits;            // down GEMM K splits
  int gu_splits;         // gate-up GEMM K splits (1: fused SiLU*up epilogue)
  int dn_bn, gu_bn;      // N tile widths
  int part_dtype;        // dtype of the down GEMM's weighted rows
  size_t align_ws;
  int sms;
  size_t off_sorted, off_eids, off_npp, off_align, off_inv, off_a, off_a_scale, off_act,
      off_act_q, off_act_scale, off_part, off_gu_part, total;
  bool token_gather;     // gather through the align's slot map (token-major)
};

int elem_bytes(int dtype) {
  switch (dtype) {
    case MOE_DTYPE_F32: case MOE_DTYPE_I32: return 4;
    case MOE_DTYPE_F16: case MOE_DTYPE_BF16: return 2;
    case MOE_DTYPE_E4M3: case MOE_DTYPE_I8: return 1;
    case MOE_DTYPE_I64: return 8;
    default: return 0;
  }
}

// MOE_NO_TOKEN_GATHER=1 keeps the row-major gather (one source read per
// routed row) in moe_fused_experts; the two write the same operand bytes.
bool token_gather_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("MOE_NO_TOKEN_GATHER");
    return !(v && v[0] && v[0] != '0');
  }();
  return on;
}

// Upper bound on the m-blocks a routing can use: an expert with c rows needs
// ceil(c / 128) <= c / 128 + 1 blocks and at most min(E, numel) experts
// have rows.
int64_t est_m_blocks(int64_t numel, int64_t L, int E) {
  return std::min<int64_t>(L / kBlockM, numel / kBlockM + std::min<int64_t>(E, numel));
}

// Tile width and K split of one grouped GEMM with `n` output columns, a
// reduction of `k_bytes` bytes per row and `rows` routed rows over `mb`
// m-blocks. Cost model in bytes moved at the whole-GPU rate:
//   waves * per-tile bytes * sms, per-tile bytes = (BN + 32) * k_bytes / S
// (a CTA streams its B tile, BN rows, plus the A tile, counted as 32 rows
// since it mostly hits L2, over its 1/S share of K; the kernel takes
// ceil(tiles * S / sms) such waves, each with a fixed start-up cost of about
// a microsecond of streaming, 48 KB), plus the split's extra traffic: S fp32
// partial rows written and read back instead of one 16-bit row
// ((8*S - 4) * rows * n bytes; S = 1 costs nothing extra).
struct Tiling {
  int bn;
  int splits;
};

Tiling choose_tiling(int64_t mb, int64_t rows, int64_t n, int64_t k_bytes, int sms,
                     bool allow_split, bool allow64, int max_bn = 256) {
  Tiling best{0, 1};
  double best_cost = 1e300;
  mb = std::max<int64_t>(mb, 1);
  const int64_t k_blocks = ceil_div(k_bytes, 128);
  for (int bn : {256, 128, 64}) {
    if (n % bn != 0 || (bn == 64 && !allow64) || bn > max_bn) continue;
    const int64_t tiles = mb * (n / bn);
    const int64_t max_s =
        allow_split ? std::min<int64_t>(16, std::max<int64_t>(1, k_blocks / 4)) : 1;
    for (int64_t s = 1; s <= max_s; ++s) {
      const int64_t per = ceil_div(k_blocks, s);
      if (ceil_div(k_blocks, per) != s) continue;  // a split would be empty
      const double waves = double(ceil_div(tiles * s, sms));
      double cost =
          waves * (double(bn + 32) * double(k_bytes) / double(s) + 48.0 * 1024.0) * double(sms);
      if (s > 1) cost += double(8 * s - 4) * double(rows) * double(n);
      if (cost < best_cost * 0.999) {
        best_cost = cost;
        best = Tiling{bn, int(s)};
      }
    }
  }
  return best;
}

int make_plan(const moe_problem_t* p, int sms, Plan* pl) {
  KSW_REQUIRE(p != nullptr, MOE_ERR_INVALID_ARG, "null problem");
  KSW_REQUIRE(p->num_tokens >= 0 && p->hidden_size > 0 && p->inter_size > 0,
              MOE_ERR_INVALID_ARG, "bad sizes");
  KSW_REQUIRE(p->num_experts >= 1 && p->num_experts <= 1024, MOE_ERR_UNSUPPORTED,
              "num_experts must be in [1, 1024]");
  KSW_REQUIRE(p->top_k >= 1 && p->top_k <= 64, MOE_ERR_INVALID_ARG, "top_k must be in [1, 64]");
  KSW_REQUIRE(p->hidden_size % 64 == 0, MOE_ERR_UNSUPPORTED,
              "hidden_size must be a multiple of 64");
  KSW_REQUIRE(p->inter_size % 16 == 0, MOE_ERR_UNSUPPORTED,
              "intermediate_size must be a multiple of 16");
  KSW_REQUIRE(p->act_dtype == MOE_DTYPE_F32 || p->act_dtype == MOE_DTYPE_F16 ||
                  p->act_dtype == MOE_DTYPE_BF16,
              MOE_ERR_INVALID_ARG, "act_dtype must be f32, f16 or bf16");
  KSW_REQUIRE(p->ids_dtype == MOE_DTYPE_I32 || p->ids_dtype == MOE_DTYPE_I64,
              MOE_ERR_INVALID_ARG, "ids_dtype must be int32 or int64");
  KSW_REQUIRE(p->weights_dtype == MOE_DTYPE_F32 || p->weights_dtype == MOE_DTYPE_F16 ||
                  p->weights_dtype == MOE_DTYPE_BF16,
              MOE_ERR_INVALID_ARG, "weights_dtype must be f32, f16 or bf16");
  Plan& P = *pl;
  P.T = p->num_tokens;
  P.H = p->hidden_size;
  P.I = p->inter_size;
  P.E = p->num_experts;
  P.k = p->top_k;
  P.quant = p->quant;
  P.numel = P.T * P.k;
  KSW_REQUIRE(P.numel < (int64_t(1) << 30), MOE_ERR_UNSUPPORTED, "too many tokens");
  P.L = align_buffer_len(P.numel, P.E, kBlockM);
  // 16-bit activations compute in their own dtype; fp32 activations keep
  // fp32 operands, multiplied as tf32 (unquantised weights), or go through
  // bf16 for the W8A8 paths
  P.compute_dtype = p->act_dtype == MOE_DTYPE_F16 ? MOE_DTYPE_F16
                    : p->act_dtype == MOE_DTYPE_F32 && p->quant == MOE_QUANT_NONE
                        ? MOE_DTYPE_F32
                        : MOE_DTYPE_BF16;
  int kbpe = 2;
  if (P.quant == MOE_QUANT_NONE) {
    P.a_dtype = P.compute_dtype;
    P.act_dtype = P.compute_dtype;
    kbpe = int(elem_bytes(P.compute_dtype));
  } else if (P.quant == MOE_QUANT_INT8_CHANNEL) {
    P.a_dtype = MOE_DTYPE_I8;
    P.act_dtype = MOE_DTYPE_BF16;
    kbpe = 1;
  } else if (P.quant == MOE_QUANT_FP8_BLOCK || P.quant == MOE_QUANT_FP8_UE8M0) {
    KSW_REQUIRE(P.I % 128 == 0 && P.H % 128 == 0, MOE_ERR_UNSUPPORTED,
                "fp8 block-scaled path needs hidden and intermediate sizes divisible by 128");
    P.a_dtype = MOE_DTYPE_E4M3;
    P.act_dtype = MOE_DTYPE_BF16;
    kbpe = 1;
  } else {
    return fail(MOE_ERR_INVALID_ARG, "unknown quant mode");
  }
  const int64_t est_mb = est_m_blocks(P.numel, P.L, P.E);
  const bool fp8 = P.quant == MOE_QUANT_FP8_BLOCK;
  const bool mx = P.quant == MOE_QUANT_FP8_UE8M0;
  const int max_bn = 256;
  // The UE8M0 kernel holds one TMEM accumulator at 256 columns and two at
  // 128, so a 128-wide down GEMM (few k-blocks per tile) overlaps each
  // tile's epilogue with the next tile's MMAs once the experts have rows to
  // fill their m-blocks (DeepSeek-V3 T=4096, 128 routed rows per expert:
  // down 1.10 -> 1.06 ms); with a few rows per expert (T=64: 2) the extra
  // tiles cost more than the overlap gains (0.54 -> 0.58 ms), and the
  // gate-up, with 56 k-blocks per tile, keeps 256.
  const int dn_max_bn = mx && P.numel >= 64 * P.E ? 128 : max_bn;
  const Tiling dn = choose_tiling(est_mb, P.numel, P.H, P.I * kbpe, sms, true, !(fp8 || mx),
                                  dn_max_bn);
  // the split gate-up path has no fp8 epilogue (its block scales follow the
  // regrouped gate/up rows); fp8 keeps the fused SiLU*up epilogue
  const Tiling gu = choose_tiling(est_mb, P.numel, 2 * P.I, P.H * kbpe, sms, !(fp8 || mx),
                                  !(fp8 || mx), max_bn);
  KSW_REQUIRE(dn.bn > 0 && gu.bn > 0, MOE_ERR_UNSUPPORTED,
              "hidden size and 2*intermediate size must be multiples of 64 (128 for fp8)");
  P.splits = dn.splits;
  P.dn_bn = dn.bn;
  P.gu_splits = gu.splits;
  P.gu_bn = gu.bn;
  // MOE_BLOCK_N=64/128/256 overrides the tile width of each GEMM it divides
  // (and that allows it: fp8 tiles are 128 or 256 wide), for timing studies
  if (const char* v = std::getenv("MOE_BLOCK_N")) {
    const int bn = std::atoi(v);
    if ((bn == 128 || bn == 256 || (bn == 64 && !fp8 && !mx)) && bn <= max_bn) {
      if (P.H % bn == 0) P.dn_bn = bn;
      if ((2 * P.I) % bn == 0) P.gu_bn = bn;
    }
  }
  // Without a K split each weighted row is final: keep it in the 16-bit
  // activation dtype (as base.py:72,75 does) and halve the row traffic;
  // K-split partial sums and fp32 activations stay fp32.
  P.part_dtype = MOE_DTYPE_F32;
  if (P.splits == 1 && !fp8 && p->act_dtype == P.compute_dtype &&
      (P.quant == MOE_QUANT_NONE || P.compute_dtype == MOE_DTYPE_BF16))
    P.part_dtype = P.compute_dtype;
  P.align_ws = align_workspace_bytes(P.numel, P.E);

  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align256(off + bytes);
    return o;
  };
  P.off_sorted = take(size_t(P.L) * 4);
  P.off_eids = take(size_t(P.L / kBlockM) * 4);
  P.off_npp = take(4);
  P.off_align = take(P.align_ws);
  // the token-major gather reads each token once and writes its top_k rows
  P.token_gather = token_gather_enabled() && P.k <= 32 &&
                   (P.quant == MOE_QUANT_NONE || P.quant == MOE_QUANT_FP8_BLOCK ||
                    P.quant == MOE_QUANT_FP8_UE8M0);
  P.off_inv = take(P.token_gather ? size_t(P.numel) * 4 : 0);
  P.off_a = take(size_t(P.L) * P.H * elem_bytes(P.a_dtype));
  // per-row scales: int8 one per row, fp8 one per row per 128 columns (fp32,
  // or one byte in the scale-factor image for UE8M0)
  auto scale_bytes = [&](int64_t cols) -> size_t {
    if (P.quant == MOE_QUANT_INT8_CHANNEL) return size_t(P.L) * 4;
    if (P.quant == MOE_QUANT_FP8_BLOCK) return size_t(P.L) * size_t(ceil_div(cols, 128)) * 4;
    if (P.quant == MOE_QUANT_FP8_UE8M0) return size_t(moe_ue8m0_scale_bytes(1, P.L, cols));
    return 0;
  };
  P.off_a_scale = take(scale_bytes(P.H));
  P.off_act = take(size_t(P.L) * P.I * elem_bytes(P.act_dtype));
  P.off_act_q = take(P.quant != MOE_QUANT_NONE ? size_t(P.L) * P.I : 0);
  P.off_act_scale = take(scale_bytes(P.I));
  P.off_part = take(size_t(P.splits) * P.numel * P.H * elem_bytes(P.part_dtype));
  P.off_gu_part = take(P.gu_splits > 1 ? size_t(P.gu_splits) * P.numel * 2 * P.I * 4 : 0);
  P.sms = sms;
  P.total = off;
  return MOE_OK;
}

template <typename T>
T* at(void* ws, size_t off) {
  return reinterpret_cast<T*>(static_cast<uint8_t*>(ws) + off);
}

}  // namespace
}  // namespace ksw

using namespace ksw;

extern "C" {

int moe_fused_experts_workspace_size(const moe_problem_t* p, size_t* bytes) {
  KSW_REQUIRE(bytes != nullptr, MOE_ERR_INVALID_ARG, "null bytes pointer");
  int sms = 148;
  int st = check_device(&sms);
  if (st != MOE_OK) sms = 148;  // size queries work without a B200 present
  Plan pl;
  st = make_plan(p, sms, &pl);
  if (st != MOE_OK) return st;
  *bytes = pl.total;
  return MOE_OK;
}

// The forward of moe_fused_experts; with `rows_out` (top_k == 1 only) the
// per-row expert outputs go straight to rows_out from the down GEMM when it
// runs unsplit, and the top-k sum is skipped. With `logits` (moe_fused_moe)
// the tokens are routed first into p->topk_weights / p->topk_ids: inside
// the decode kernel when it runs and the logits are fp32 over at most 256
// experts, else by moe_topk_softmax.
static int fused_experts_impl(const moe_problem_t* p, void* workspace, size_t workspace_bytes,
                              void* stream, void* rows_out, const void* logits = nullptr,
                              int logits_dtype = MOE_DTYPE_F32, int renorm = 1) {
  // 16-byte vectors and bulk copies: a misaligned operand would fault the
  // context, so it is refused here, before the device is touched
  // (fp8 128x128 block scales are read one float at a time)
  KSW_REQUIRE(p != nullptr, MOE_ERR_INVALID_ARG, "null problem");
  const bool vec_scales = p->quant != MOE_QUANT_FP8_BLOCK;
  KSW_REQUIRE(aligned16(p->hidden) && aligned16(p->w13) && aligned16(p->w2) &&
                  aligned16(p->out) && aligned16(rows_out) && aligned16(workspace) &&
                  (!vec_scales || (aligned16(p->w13_scale) && aligned16(p->w2_scale))),
              MOE_ERR_INVALID_ARG,
              "moe_fused_experts: hidden, w13, w2, out, workspace and the int8 / UE8M0 "
              "weight scales must be 16-byte aligned");
  int sms = 0;
  int st = check_device(&sms);
  if (st != MOE_OK) return st;
  Plan P;
  st = make_plan(p, sms, &P);
  if (st != MOE_OK) return st;
  KSW_REQUIRE(workspace != nullptr && workspace_bytes >= P.total, MOE_ERR_WORKSPACE,
              "moe_fused_experts: workspace smaller than moe_fused_experts_workspace_size");
  if (P.T == 0) return MOE_OK;
  KSW_REQUIRE(p->out != nullptr, MOE_ERR_INVALID_ARG, "null out");
  KSW_REQUIRE(p->hidden && p->w13 && p->w2 && p->topk_weights && p->topk_ids,
              MOE_ERR_INVALID_ARG, "null input pointer");
  if (P.quant != MOE_QUANT_NONE)
    KSW_REQUIRE(p->w13_scale && p->w2_scale, MOE_ERR_INVALID_ARG, "null weight scales");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool decode = P.quant == MOE_QUANT_NONE && p->act_dtype == P.compute_dtype &&
                      p->num_tokens_dev == nullptr && decode_path_enabled() &&
                      decode_path_fits(P.T, P.k, P.H, P.I, p->act_dtype);
  // fp32 logits over at most 256 experts on the decode path: the decode
  // gate-up kernel routes the tokens itself (one launch fewer)
  const bool route_in_decode = logits != nullptr && decode && logits_dtype == MOE_DTYPE_F32 &&
                               P.E <= kDecodeRouteMaxExperts;
  if (logits != nullptr && !route_in_decode) {
    st = moe_topk_softmax(logits, logits_dtype, P.T, P.E, P.k, renorm,
                          const_cast<void*>(p->topk_weights), p->weights_dtype,
                          const_cast<void*>(p->topk_ids), p->ids_dtype, stream);
    if (st != MOE_OK) return st;
  }
  // Stage events: inside a stream capture they become event-record nodes of
  // the graph (external records), so a replayed graph can be timed per stage.
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (p->stage_events != nullptr)
    KSW_CUDA(cudaStreamIsCapturing(s, &cap));
  auto mark = [&](int stage) -> int {
    if (p->stage_events == nullptr) return MOE_OK;
    cudaEvent_t ev = static_cast<cudaEvent_t>(p->stage_events[stage]);
    if (cap == cudaStreamCaptureStatusActive)
      return check_cuda(cudaEventRecordWithFlags(ev, s, cudaEventRecordExternal),
                        "cudaEventRecordWithFlags(stage event)");
    return check_cuda(cudaEventRecord(ev, s), "cudaEventRecord(stage event)");
  };
#define KSW_MARK(stage)           \
  do {                            \
    st = mark(stage);             \
    if (st != MOE_OK) return st;  \
  } while (0)
  // A handful of routed rows with 16-bit operands: stream the weights
  // through the two decode kernels (csrc/decode.cu).
  if (decode) {
    DecodeArgs d{};
    d.T = P.T;
    d.H = P.H;
    d.I = P.I;
    d.top_k = P.k;
    d.E = P.E;
    d.act_dtype = p->act_dtype;
    d.ids_dtype = p->ids_dtype;
    d.weights_dtype = p->weights_dtype;
    d.hidden = p->hidden;
    d.w13 = p->w13;
    d.w2 = p->w2;
    d.ids = p->topk_ids;
    d.weights = p->topk_weights;
    d.act = at<void>(workspace, P.off_act);
    d.out = rows_out != nullptr ? rows_out : p->out;
    d.logits = route_in_decode ? logits : nullptr;
    d.renorm = renorm;
    KSW_MARK(MOE_STAGE_ALIGN);
    KSW_MARK(MOE_STAGE_GATHER);
    KSW_MARK(MOE_STAGE_GATE_UP);
    st = decode_launch(d, 0, s);
    if (st != MOE_OK) return st;
    KSW_MARK(MOE_STAGE_QUANT);
    KSW_MARK(MOE_STAGE_DOWN);
    st = decode_launch(d, 1, s);
    if (st != MOE_OK) return st;
    KSW_MARK(MOE_STAGE_SUM);
    KSW_MARK(MOE_NUM_STAGES);
    return MOE_OK;
  }

  int32_t* sorted = at<int32_t>(workspace, P.off_sorted);
  int32_t* eids = at<int32_t>(workspace, P.off_eids);
  int32_t* npp = at<int32_t>(workspace, P.off_npp);

  KSW_MARK(MOE_STAGE_ALIGN);
  int32_t* inv = P.token_gather ? at<int32_t>(workspace, P.off_inv) : nullptr;
  st = align_launch(p->topk_ids, p->ids_dtype, P.numel, P.E, kBlockM, sorted, eids, npp,
                    at<void>(workspace, P.off_align), P.align_ws, s, p->num_tokens_dev, P.k,
                    inv);
  if (st != MOE_OK) return st;

  GatherArgs g{};
  g.src = p->hidden;
  g.src_dtype = p->act_dtype;
  g.src_rows = P.T;
  g.H = P.H;
  g.top_k = P.k;
  g.sorted = sorted;
  g.num_post_pad = npp;
  g.max_rows = P.L;
  g.numel = P.numel;
  g.quant = P.quant;
  g.dst = at<void>(workspace, P.off_a);
  g.dst_dtype = P.a_dtype;
  g.scale = P.quant == MOE_QUANT_NONE ? nullptr : at<float>(workspace, P.off_a_scale);
  g.inv = inv;
  g.src_count = p->num_tokens_dev;
  KSW_MARK(MOE_STAGE_GATHER);
  st = gather_launch(g, s);
  if (st != MOE_OK) return st;

  KSW_MARK(MOE_STAGE_GATE_UP);
  GroupedGemmArgs ga{};
  ga.quant = P.quant;
  ga.compute_dtype = P.compute_dtype;
  ga.a = g.dst;
  ga.a_scale = g.scale;
  ga.b = p->w13;
  ga.b_scale = p->w13_scale;
  ga.sorted_ids = sorted;
  ga.expert_ids = eids;
  ga.num_post_pad = npp;
  ga.rows = P.L;
  ga.numel = P.numel;
  ga.num_experts = P.E;
  ga.n = 2 * P.I;
  ga.k = P.H;
  ga.out = at<void>(workspace, P.off_act);
  ga.splits = 1;
  ga.status = p->status;
  ga.early_meta = 1;  // align ran two launches earlier (the gather is between)
  if (P.gu_splits > 1) {
    // decode-sized: split K, unweighted fp32 partial rows, then SiLU*up
    GroupedGemmArgs gs = ga;
    gs.out = at<void>(workspace, P.off_gu_part);
    gs.splits = P.gu_splits;
    gs.block_n = P.gu_bn;
    st = gemm_gate_up_split_launch(gs, s);
    if (st != MOE_OK) return st;
    st = swiglu_reduce_launch(at<float>(workspace, P.off_gu_part), P.gu_splits, P.numel, P.I,
                              sorted, npp, P.L, ga.out, P.act_dtype, s);
  } else {
    ga.block_n = P.gu_bn;
    st = gemm_gate_up_launch(ga, s);
  }
  if (st != MOE_OK) return st;

  const void* down_a = ga.out;
  const float* down_a_scale = nullptr;
  KSW_MARK(MOE_STAGE_QUANT);
  if (P.quant != MOE_QUANT_NONE) {
    GatherArgs q{};
    q.src = ga.out;
    q.src_dtype = P.act_dtype;
    q.src_rows = P.L;
    q.H = P.I;
    q.top_k = 0;
    q.sorted = sorted;
    q.num_post_pad = npp;
    q.max_rows = P.L;
    q.numel = P.numel;
    q.quant = P.quant;
    q.dst = at<void>(workspace, P.off_act_q);
    q.dst_dtype = P.a_dtype;
    q.scale = at<float>(workspace, P.off_act_scale);
    st = gather_launch(q, s);
    if (st != MOE_OK) return st;
    down_a = q.dst;
    down_a_scale = q.scale;
  }

  KSW_MARK(MOE_STAGE_DOWN);
  GroupedGemmArgs gd = ga;
  gd.a = down_a;
  gd.a_scale = down_a_scale;
  gd.b = p->w2;
  gd.b_scale = p->w2_scale;
  gd.n = P.H;
  gd.k = P.I;
  gd.out = at<void>(workspace, P.off_part);
  gd.row_weights = p->topk_weights;
  gd.row_weights_dtype = p->weights_dtype;
  gd.splits = P.splits;
  gd.block_n = P.dn_bn;
  gd.out_dtype = P.part_dtype;
  const bool direct = rows_out != nullptr && P.splits == 1 && P.part_dtype == p->act_dtype;
  if (direct) gd.out = rows_out;  // weighted rows in token order: the result itself
  st = gemm_down_launch(gd, s);
  if (st != MOE_OK) return st;
  if (direct) {
    KSW_MARK(MOE_STAGE_SUM);
    KSW_MARK(MOE_NUM_STAGES);
    return MOE_OK;
  }

  SumArgs sa{};
  sa.part = at<void>(workspace, P.off_part);
  sa.part_dtype = P.part_dtype;
  sa.splits = P.splits;
  sa.T = P.T;
  sa.top_k = P.k;
  sa.H = P.H;
  sa.ids = p->topk_ids;
  sa.ids_dtype = p->ids_dtype;
  sa.E = P.E;
  sa.out = rows_out != nullptr ? rows_out : p->out;
  sa.out_dtype = p->act_dtype;
  sa.count_dev = p->num_tokens_dev;
  KSW_MARK(MOE_STAGE_SUM);
  st = sum_topk_launch(sa, s);
  if (st != MOE_OK) return st;
  KSW_MARK(MOE_NUM_STAGES);
  return MOE_OK;
#undef KSW_MARK
}

int moe_fused_experts(const moe_problem_t* p, void* workspace, size_t workspace_bytes,
                      void* stream) {
  return fused_experts_impl(p, workspace, workspace_bytes, stream, nullptr);
}

int moe_fused_moe(const moe_problem_t* p, const void* router_logits, int logits_dtype,
                  int renormalize, void* workspace, size_t workspace_bytes, void* stream) {
  KSW_REQUIRE(router_logits != nullptr, MOE_ERR_INVALID_ARG, "moe_fused_moe: null logits");
  KSW_REQUIRE(logits_dtype == MOE_DTYPE_F32 || logits_dtype == MOE_DTYPE_F16 ||
                  logits_dtype == MOE_DTYPE_BF16,
              MOE_ERR_INVALID_ARG, "moe_fused_moe: logits must be f32, f16 or bf16");
  return fused_experts_impl(p, workspace, workspace_bytes, stream, nullptr, router_logits,
                            logits_dtype, renormalize ? 1 : 0);
}

int moe_fused_moe_launches(const moe_problem_t* p, int logits_dtype, int* launches) {
  KSW_REQUIRE(launches != nullptr, MOE_ERR_INVALID_ARG, "null launches pointer");
  int n = 0;
  int st = moe_fused_experts_launches(p, 0, &n);
  if (st != MOE_OK) return st;
  if (n == 0) {
    *launches = 0;
    return MOE_OK;
  }
  int sms = 148;
  if (check_device(&sms) != MOE_OK) sms = 148;
  Plan P;
  st = make_plan(p, sms, &P);
  if (st != MOE_OK) return st;
  const bool decode = P.quant == MOE_QUANT_NONE && p->act_dtype == P.compute_dtype &&
                      p->num_tokens_dev == nullptr && decode_path_enabled() &&
                      decode_path_fits(P.T, P.k, P.H, P.I, p->act_dtype);
  const bool routed_inside = decode && logits_dtype == MOE_DTYPE_F32 &&
                             P.E <= kDecodeRouteMaxExperts;
  *launches = n + (routed_inside ? 0 : 1);
  return MOE_OK;
}

int moe_fused_experts_launches(const moe_problem_t* p, int rows_only, int* launches) {
  KSW_REQUIRE(launches != nullptr, MOE_ERR_INVALID_ARG, "null launches pointer");
  int sms = 148;
  if (check_device(&sms) != MOE_OK) sms = 148;  // answers without a B200 present
  Plan P;
  const int st = make_plan(p, sms, &P);
  if (st != MOE_OK) return st;
  if (P.T == 0) {
    *launches = 0;
    return MOE_OK;
  }
  if (P.quant == MOE_QUANT_NONE && p->act_dtype == P.compute_dtype &&
      p->num_tokens_dev == nullptr && decode_path_enabled() &&
      decode_path_fits(P.T, P.k, P.H, P.I, p->act_dtype)) {
    *launches = 2;  // the two decode kernels
    return MOE_OK;
  }
  int n = (P.numel <= align_small_max() ? 1 : 3);      // align
  n += 1;                                               // gather
  n += P.gu_splits > 1 ? 2 : 1;                         // gate-up (+ swiglu_reduce)
  n += P.quant != MOE_QUANT_NONE ? 1 : 0;               // activation quantisation
  n += 1;                                               // down
  const bool direct = rows_only && p->top_k == 1 && P.splits == 1 && P.part_dtype == p->act_dtype;
  n += direct ? 0 : 1;                                  // top-k sum
  *launches = n;
  return MOE_OK;
}

int moe_fused_experts_plan(const moe_problem_t* p, int32_t* info) {
  KSW_REQUIRE(info != nullptr, MOE_ERR_INVALID_ARG, "null info pointer");
  int sms = 148;
  if (check_device(&sms) != MOE_OK) sms = 148;  // answers without a B200 present
  Plan P;
  const int st = make_plan(p, sms, &P);
  if (st != MOE_OK) return st;
  const bool decode = P.quant == MOE_QUANT_NONE && p->act_dtype == P.compute_dtype &&
                      p->num_tokens_dev == nullptr && decode_path_enabled() &&
                      decode_path_fits(P.T, P.k, P.H, P.I, p->act_dtype);
  info[0] = P.gu_bn;
  info[1] = P.gu_splits;
  info[2] = P.dn_bn;
  info[3] = P.splits;
  info[4] = P.part_dtype;
  info[5] = !decode && P.token_gather ? 1 : 0;
  info[6] = decode ? 1 : 0;
  info[7] = sms;
  return MOE_OK;
}

int moe_fused_experts_rows(const moe_problem_t* p, void* workspace, size_t workspace_bytes,
                           void* stream) {
  KSW_REQUIRE(p != nullptr, MOE_ERR_INVALID_ARG, "null problem");
  KSW_REQUIRE(p->top_k == 1, MOE_ERR_INVALID_ARG, "moe_fused_experts_rows: top_k must be 1");
  return fused_experts_impl(p, workspace, workspace_bytes, stream, p->out);
}

int moe_gather_rows(const void* src, int src_dtype, int64_t src_rows, int64_t hidden_size,
                    int top_k, const int32_t* sorted_token_ids,
                    const int32_t* num_tokens_post_pad, int64_t buffer_len, int64_t numel,
                    int quant, void* dst, int dst_dtype, float* dst_scale, void* stream) {
  int st = check_device(nullptr);
  if (st != MOE_OK) return st;
  GatherArgs g{};
  g.src = src;
  g.src_dtype = src_dtype;
  g.src_rows = src_rows;
  g.H = hidden_size;
  g.top_k = top_k;
  g.sorted = sorted_token_ids;
  g.num_post_pad = num_tokens_post_pad;
  g.max_rows = buffer_len;
  g.numel = numel;
  g.quant = quant;
  g.dst = dst;
  g.dst_dtype = dst_dtype;
  g.scale = dst_scale;
  return gather_launch(g, static_cast<cudaStream_t>(stream));
}

int moe_gemm_gate_up(int quant, int compute_dtype, const void* a, const float* a_scale,
                     const void* w13, const float* w13_scale,
                     const int32_t* sorted_token_ids, const int32_t* expert_ids,
                     const int32_t* num_tokens_post_pad, int64_t buffer_len, int64_t numel,
                     int num_experts, int64_t hidden_size, int64_t inter_size,
                     void* act_out, int block_n, int32_t* status, void* stream) {
  GroupedGemmArgs ga{};
  ga.quant = quant;
  ga.compute_dtype = compute_dtype;
  ga.a = a;
  ga.a_scale = a_scale;
  ga.b = w13;
  ga.b_scale = w13_scale;
  ga.sorted_ids = sorted_token_ids;
  ga.expert_ids = expert_ids;
  ga.num_post_pad = num_tokens_post_pad;
  ga.rows = buffer_len;
  ga.numel = numel;
  ga.num_experts = num_experts;
  ga.n = 2 * inter_size;
  ga.k = hidden_size;
  ga.out = act_out;
  ga.splits = 1;
  ga.status = status;
  ga.block_n = block_n;
  return gemm_gate_up_launch(ga, static_cast<cudaStream_t>(stream));
}

int moe_gemm_down(int quant, int compute_dtype, const void* act, const float* act_scale,
                  const void* w2, const float* w2_scale, const int32_t* sorted_token_ids,
                  const int32_t* expert_ids, const int32_t* num_tokens_post_pad,
                  int64_t buffer_len, int64_t numel, int num_experts, int64_t hidden_size,
                  int64_t inter_size, const void* row_weights, int weights_dtype, int splits,
                  float* partial_out, int block_n, int32_t* status, void* stream) {
  GroupedGemmArgs gd{};
  gd.quant = quant;
  gd.compute_dtype = compute_dtype;
  gd.a = act;
  gd.a_scale = act_scale;
  gd.b = w2;
  gd.b_scale = w2_scale;
  gd.sorted_ids = sorted_token_ids;
  gd.expert_ids = expert_ids;
  gd.num_post_pad = num_tokens_post_pad;
  gd.rows = buffer_len;
  gd.numel = numel;
  gd.num_experts = num_experts;
  gd.n = hidden_size;
  gd.k = inter_size;
  gd.out = partial_out;
  gd.row_weights = row_weights;
  gd.row_weights_dtype = weights_dtype;
  gd.splits = splits;
  gd.status = status;
  gd.block_n = block_n;
  return gemm_down_launch(gd, static_cast<cudaStream_t>(stream));
}

int moe_sum_topk(const float* partial, int splits, int64_t num_tokens, int top_k,
                 int64_t hidden_size, const void* topk_ids, int ids_dtype, int num_experts,
                 void* out, int out_dtype, void* stream) {
  int st = check_device(nullptr);
  if (st != MOE_OK) return st;
  SumArgs sa{};
  sa.part = partial;
  sa.part_dtype = MOE_DTYPE_F32;
  sa.splits = splits;
  sa.T = num_tokens;
  sa.top_k = top_k;
  sa.H = hidden_size;
  sa.ids = topk_ids;
  sa.ids_dtype = ids_dtype;
  sa.E = num_experts;
  sa.out = out;
  sa.out_dtype = out_dtype;
  return sum_topk_launch(sa, static_cast<cudaStream_t>(stream));
}

int moe_combine_rows(const void* rows, int rows_dtype, const int32_t* inv_index,
                     const void* weights, int weights_dtype, int64_t num_tokens, int top_k,
                     int64_t hidden_size, void* out, int out_dtype, void* stream) {
  int st = check_device(nullptr);
  if (st != MOE_OK) return st;
  CombineArgs c{};
  c.rows = rows;
  c.rows_dtype = rows_dtype;
  c.inv = inv_index;
  c.weights = weights;
  c.weights_dtype = weights_dtype;
  c.T = num_tokens;
  c.top_k = top_k;
  c.H = hidden_size;
  c.out = out;
  c.out_dtype = out_dtype;
  return combine_launch(c, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
