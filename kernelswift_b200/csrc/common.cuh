// Device helpers shared by the fused-MoE kernels: host-side status plumbing,
// inline-PTX wrappers for mbarriers, TMA (cp.async.bulk.tensor), tcgen05
// tensor-memory MMA, and bounded waits that report a timeout instead of
// hanging.
#pragma once

#include <cstdint>
#include <cstdio>
#include <string>
#include <utility>

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include "../../include/moe_b200.h"

namespace ksw {

// ---------------------------------------------------------------------------
// Host-side status helpers
// ---------------------------------------------------------------------------

void set_last_error(const std::string& msg);
int fail(int status, const std::string& msg);
int check_cuda(cudaError_t err, const char* what);
// Returns MOE_OK when the current device is an sm_100 part, else an error.
int check_device(int* num_sms);

#define KSW_CUDA(call)                                        \
  do {                                                        \
    int _st = ::ksw::check_cuda((call), #call);               \
    if (_st != MOE_OK) return _st;                            \
  } while (0)

#define KSW_REQUIRE(cond, status, msg)                        \
  do {                                                        \
    if (!(cond)) return ::ksw::fail((status), (msg));         \
  } while (0)

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline int64_t round_up(int64_t a, int64_t b) { return ceil_div(a, b) * b; }
inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }
inline bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; }

// Default wait limit for on-chip barrier waits: one second.
constexpr uint64_t kWaitLimitNs = 1000ull * 1000ull * 1000ull;

// ---------------------------------------------------------------------------
// Programmatic dependent launch
//
// Every kernel of the forward is launched with programmatic stream
// serialisation, so it may start while the previous kernel in the stream is
// still running. Each kernel therefore
//   * calls pdl_wait() before it reads anything the previous kernel writes or
//     writes anything the previous kernel reads or writes, and
//   * calls pdl_trigger() only after its own pdl_wait().
// The second rule makes the ordering transitive: when kernel n starts,
// kernel n-1 has passed its wait, so kernel n-2 and everything before it
// have completed. Kernel n may therefore read the outputs of kernel n-2 and
// earlier (the align metadata, the weights) before its own wait.
// MOE_NO_PDL=1 in the environment launches everything plainly.
// ---------------------------------------------------------------------------

__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

bool pdl_enabled();

#define KSW_LAUNCH(...)                                       \
  do {                                                        \
    int _st = ::ksw::launch(__VA_ARGS__);                     \
    if (_st != MOE_OK) return _st;                            \
  } while (0)

// Launches `kern` on `s`, with programmatic stream serialisation unless
// disabled.
template <typename... KArgs, typename... Args>
int launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
           Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return check_cuda(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...),
                    "cudaLaunchKernelEx");
}

// ---------------------------------------------------------------------------
// Generic device helpers
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// Records `code` in the optional device status word (first error wins).
__device__ __forceinline__ void report_status(int32_t* status, int32_t code) {
  if (status != nullptr) atomicCAS(status, 0, code);
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar,
                                                      uint32_t bytes) {
  asm volatile(
      "mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// try_wait with a suspend-time hint: a thread whose phase is not complete
// is parked by the hardware until it completes or the hint (1 ms) passes,
// instead of polling the barrier's shared-memory word in a tight loop (which
// takes shared-memory bandwidth from the loads and the bulk copies it waits
// for). The callers re-check their time limit and abort flag between calls.
constexpr uint32_t kMbarSuspendHintNs = 1000000;

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "n"(kMbarSuspendHintNs)
      : "memory");
  return ok != 0;
}

// Waits for the phase of `bar` with parity `parity` to complete. Gives up
// when `*abort` becomes non-zero (another role gave up) or when `limit_ns`
// nanoseconds pass; in the latter case it raises `*abort` itself. Returns
// true when the phase completed.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar,
                                                  uint32_t parity,
                                                  volatile int* abort,
                                                  uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (globaltimer_ns() - t0 > limit_ns) {
      *abort = 1;
      return false;
    }
  }
}

// ---------------------------------------------------------------------------
// TMA
// ---------------------------------------------------------------------------

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* tm) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tm))
               : "memory");
}

// 2-D tiled load of the box at (c0 = inner/column, c1 = row) into shared
// memory; completion is signalled on `bar` as transaction bytes.
__device__ __forceinline__ void tma_load_2d(void* smem_dst,
                                            const CUtensorMap* tm, int32_t c0,
                                            int32_t c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::"
      "bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(c1),
      "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05 (tensor memory + 5th-generation tensor core MMA)
// ---------------------------------------------------------------------------

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile(
      "tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
          smem_u32(dst_smem)),
      "r"(ncols)
      : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::
                   : "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(
                   taddr),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Arrives once on `bar` when every tcgen05 operation this thread issued
// before the commit has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
      "[%0];" ::"r"(smem_u32(bar))
      : "memory");
}

// MMA kinds used here.
enum MmaKind : int { kKindF16 = 0, kKindF8 = 1, kKindI8 = 2, kKindTF32 = 3 };

// D[tmem] (+)= A[smem] * B[smem]^T, both operands K-major.
template <int KIND>
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc,
                                       uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  if constexpr (KIND == kKindF16) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(
            d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else if constexpr (KIND == kKindF8) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(
            d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else if constexpr (KIND == kKindTF32) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(
            d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(
            d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  }
}

// Instruction descriptor (32 bits) for a dense MMA with K-major A and B:
//   [4,6) D format (1 = f32, 2 = s32), [7,10) A format, [10,13) B format,
//   [15] A major, [16] B major (0 = K-major), [17,23) N >> 3, [24,29) M >> 4.
// A/B format: kind::f16 -> 0 f16, 1 bf16; kind::tf32 -> 2 tf32;
// kind::f8f6f4 -> 0 e4m3; kind::i8 -> 1 signed.
__host__ __device__ constexpr uint32_t make_idesc(uint32_t d_fmt,
                                                  uint32_t ab_fmt, int m,
                                                  int n) {
  return (d_fmt << 4) | (ab_fmt << 7) | (ab_fmt << 10) |
         (uint32_t(n >> 3) << 17) | (uint32_t(m >> 4) << 24);
}

// Shared-memory matrix descriptor for a K-major tile written by TMA with
// 128-byte swizzling: rows of 128 bytes, 8-row (1024-byte) swizzle atoms.
//   [0,14) start address >> 4, [16,30) leading byte offset >> 4 (unused for
//   swizzled K-major, set to 1), [32,46) stride byte offset >> 4 (1024 B
//   between 8-row groups), [46,48) version = 1, [61,64) layout = 2
//   (SWIZZLE_128B). The tile base must be 1024-byte aligned; stepping along
//   K inside the 128-byte row adds the byte offset to the start address.
__device__ __forceinline__ uint64_t make_sw128_desc(uint32_t smem_addr) {
  return (uint64_t((smem_addr >> 4) & 0x3FFFu)) | (uint64_t(1) << 16) |
         (uint64_t(1024 >> 4) << 32) | (uint64_t(1) << 46) |
         (uint64_t(2) << 61);
}

// Asks L2 to fetch `bytes` (a multiple of 16) of global memory starting at a
// 16-byte aligned address; no data reaches the thread and nothing waits.
__device__ __forceinline__ void l2_prefetch_bulk(const void* gsrc, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(
                   reinterpret_cast<uint64_t>(gsrc)),
               "r"(bytes));
}

// ----- block-scaled fp8 (kind::mxf8f6f4 with UE8M0 scale factors) -----

// 1-D bulk copy global -> shared memory, completion counted on `bar` as
// transaction bytes. Both addresses 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, "
      "[%3];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(gsrc)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Instruction descriptor of tcgen05.mma kind::mxf8f6f4.block_scale with
// e4m3 A and B (both K-major), UE8M0 scale factors and an f32 accumulator:
//   [4,6) B scale-factor byte, [7,10) A format 0 (e4m3), [10,13) B format 0,
//   [17,23) N >> 3, [23] scale format 1 (UE8M0), [24,29) M >> 4,
//   [29,31) A scale-factor byte, [31] K = 32.
__host__ __device__ constexpr uint32_t make_idesc_mx(int m, int n) {
  return (uint32_t(n >> 3) << 17) | (1u << 23) | (uint32_t(m >> 4) << 24);
}
// Selects byte `id` (0..3) of the 32-bit scale-factor cells for A and B.
__host__ __device__ constexpr uint32_t idesc_sf_ids(uint32_t idesc, uint32_t id) {
  return idesc | (id << 29) | (id << 4);
}

// D[tmem] (+)= (A * sfA) * (B * sfB)^T for one K = 32 step: the scale
// factor of A row m and of B row n live in tensor memory at sfa_tmem /
// sfb_tmem (layout of tc_cp_sf below).
__device__ __forceinline__ void tc_mma_mx(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t sfa_tmem,
                                          uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], "
      "p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

// Copies a 512-byte scale-factor chunk (32 rows of 16 bytes in shared
// memory) into tensor memory: row l goes to lane l of the four columns at
// `taddr`, replicated into each of the four 32-lane quarters. A chunk holds
// the scales of 128 matrix rows: row r's four bytes (four consecutive
// k-blocks) are the 32-bit cell of lane r % 32, column r / 32.
__device__ __forceinline__ void tc_cp_sf(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc)
               : "memory");
}

// Shared-memory descriptor of one scale-factor chunk: no swizzle, 8-row x
// 16-byte core matrices stored contiguously (stride byte offset 128 between
// them), one core matrix across, version 1.
__device__ __forceinline__ uint64_t make_sf_desc(uint32_t smem_addr) {
  return (uint64_t((smem_addr >> 4) & 0x3FFFu)) | (uint64_t(128 >> 4) << 32) |
         (uint64_t(1) << 46);
}

// UE8M0 scale byte of a group with absolute maximum `amax`: the smallest b
// with amax <= 448 * 2^(b - 127). Writing amax = 1.f * 2^(E - 127) (f the
// 23-bit fraction, E the biased exponent): 448 = 1.75 * 2^8, so b = E - 8
// when 1.f <= 1.75 and E - 7 otherwise. Zero (and NaN) groups get 127
// (scale 1); subnormal groups get 0.
__device__ __forceinline__ uint32_t ue8m0_byte(float amax) {
  if (!(amax > 0.0f)) return 127u;
  const uint32_t bits = __float_as_uint(amax);
  const int b = int((bits >> 23) & 0xFFu) - 8 + ((bits & 0x7FFFFFu) > 0x600000u ? 1 : 0);
  return uint32_t(min(max(b, 0), 254));
}
// 1 / scale = 2^(127 - b), exactly (b <= 253).
__device__ __forceinline__ float ue8m0_inv_scale(uint32_t b) {
  return __uint_as_float((254u - b) << 23);
}

// fp32 -> tf32 (10 mantissa bits), round to nearest, ties away from zero;
// the low 13 bits of the result are zero. The tf32 GEMMs take operands
// rounded this way (the tensor core itself ignores the low bits).
__device__ __forceinline__ float round_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

constexpr float kFp8Max = 448.0f;

// Two values -> two e4m3 bytes (low byte = first value): x * inv clamped to
// +-448, rounded to nearest even.
__device__ __forceinline__ uint32_t to_e4m3x2(float x0, float x1, float inv) {
  const float q0 = fminf(fmaxf(x0 * inv, -kFp8Max), kFp8Max);
  const float q1 = fminf(fmaxf(x1 * inv, -kFp8Max), kFp8Max);
  return uint32_t(__nv_cvt_float2_to_fp8x2(make_float2(q0, q1), __NV_SATFINITE, __NV_E4M3));
}

// Eight values -> eight e4m3 bytes in column order.
__device__ __forceinline__ uint2 pack_e4m3x8(const float (&v)[8], float inv) {
  const uint32_t lo = to_e4m3x2(v[0], v[1], inv) | (to_e4m3x2(v[2], v[3], inv) << 16);
  const uint32_t hi = to_e4m3x2(v[4], v[5], inv) | (to_e4m3x2(v[6], v[7], inv) << 16);
  return make_uint2(lo, hi);
}

// Byte offset of the scale of row r, column block kb in a scale-factor image
// with q_blocks = ceil(KB / 4) and row_slices = ceil(R / 128), for matrix
// group g (the layout moe_ue8m0_scale_bytes documents).
__host__ __device__ __forceinline__ int64_t sf_image_offset(int64_t g, int64_t r, int64_t kb,
                                                            int64_t q_blocks,
                                                            int64_t row_slices) {
  return ((g * q_blocks + (kb >> 2)) * row_slices + (r >> 7)) * 512 + 16 * (r & 31) +
         4 * ((r & 127) >> 5) + (kb & 3);
}

// Loads 16 consecutive 32-bit columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]),
        "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]),
        "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15])
      : "r"(taddr));
}

// Loads 4 consecutive 32-bit columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, uint32_t (&r)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Element conversion helpers
// ---------------------------------------------------------------------------

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) {
  return __half2float(v);
}
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) {
  return __float2half_rn(v);
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// Register re-allocation between warpgroups (all four warps of a warpgroup
// execute it together).
template <int N>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// Packs two floats into one 32-bit word of two 16-bit elements (lo first).
template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

}  // namespace ksw
