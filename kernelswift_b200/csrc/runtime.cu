// Host runtime of the C ABI: status strings, the thread-local error message,
// device checks, the device status word, TMA tensor-map encoding and the
// bounded-wait self-test kernel.
#include <cstdlib>
#include <mutex>
#include <string>

#include "common.cuh"
#include "runtime.h"

namespace ksw {

namespace {
thread_local std::string g_last_error;

// Per-device cache of the SM count and architecture check (the only global
// state of the library; written once per device under a mutex).
constexpr int kMaxDevices = 64;
std::mutex g_dev_mu;
int g_dev_sms[kMaxDevices] = {0};
int g_dev_ok[kMaxDevices] = {0};  // 0 unknown, 1 sm_100, -1 other

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t,
                                   void*, const cuuint64_t*, const cuuint64_t*,
                                   const cuuint32_t*, const cuuint32_t*,
                                   CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;
std::once_flag g_encode_once;
}  // namespace

void set_last_error(const std::string& msg) { g_last_error = msg; }

int fail(int status, const std::string& msg) {
  g_last_error = msg;
  return status;
}

int check_cuda(cudaError_t err, const char* what) {
  if (err == cudaSuccess) return MOE_OK;
  g_last_error = std::string(what) + ": " + cudaGetErrorName(err) + " (" +
                 cudaGetErrorString(err) + ")";
  return MOE_ERR_CUDA;
}

int check_device(int* num_sms) {
  int dev = 0;
  KSW_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices)
    return fail(MOE_ERR_DEVICE, "device ordinal out of range");
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (g_dev_ok[dev] == 0) {
    cudaDeviceProp prop;
    KSW_CUDA(cudaGetDeviceProperties(&prop, dev));
    g_dev_ok[dev] = (prop.major == 10 && prop.minor == 0) ? 1 : -1;
    g_dev_sms[dev] = prop.multiProcessorCount;
  }
  if (g_dev_ok[dev] != 1)
    return fail(MOE_ERR_DEVICE,
                "this library holds sm_100a code only; the current device is "
                "not a compute capability 10.0 GPU");
  if (num_sms) *num_sms = g_dev_sms[dev];
  return MOE_OK;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("MOE_NO_PDL");
    return !(v && v[0] && v[0] != '0');
  }();
  return on;
}

int encode_tma_2d(CUtensorMap* tm, CUtensorMapDataType dtype, int elem_bytes,
                  const void* base, uint64_t inner, uint64_t rows,
                  uint64_t row_stride_elems, uint32_t box_inner,
                  uint32_t box_rows) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn,
                                cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  });
  if (g_encode == nullptr)
    return fail(MOE_ERR_CUDA, "cuTensorMapEncodeTiled entry point not found");
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    return fail(MOE_ERR_INVALID_ARG, "TMA base address not 16-byte aligned");
  if ((row_stride_elems * elem_bytes) % 16 != 0)
    return fail(MOE_ERR_INVALID_ARG, "TMA row stride not a multiple of 16 B");
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {row_stride_elems * uint64_t(elem_bytes)};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(tm, dtype, 2, const_cast<void*>(base), dims, strides,
                        box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(MOE_ERR_CUDA, "cuTensorMapEncodeTiled failed with CUresult " +
                                  std::to_string(int(r)));
  return MOE_OK;
}

// One CTA, one mbarrier that nobody arrives on: the wait must run out.
__global__ void selftest_wait_kernel(int32_t* status, uint64_t limit_ns) {
  __shared__ alignas(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    bool ok = mbar_wait_bounded(&bar, 0, &abort_flag, limit_ns);
    if (!ok) report_status(status, MOE_ERR_TIMEOUT);
  }
  __syncthreads();
}

// Copies one 512-byte scale-factor chunk into tensor memory the way the
// block-scaled GEMM does (shared memory, tcgen05.cp 32x128b.warpx4) and reads
// all 128 lanes of the four columns back: out[lane * 4 + c].
__global__ void __launch_bounds__(128, 1)
    selftest_sf_copy_kernel(const uint32_t* __restrict__ chunk, uint32_t* __restrict__ out,
                            int32_t* status, uint64_t limit_ns) {
  __shared__ alignas(128) uint32_t s_chunk[128];
  __shared__ alignas(8) uint64_t bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  s_chunk[threadIdx.x] = chunk[threadIdx.x];
  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  // the copy reads shared memory through the async proxy
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  if (warp == 0) {
    tmem_alloc(&tmem_slot, 32);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tmem_slot;
  if (threadIdx.x == 0) {
    tc_cp_sf(tbase, make_sf_desc(smem_u32(s_chunk)));
    tc_commit(&bar);
  }
  const bool ok = mbar_wait_bounded(&bar, 0, &abort_flag, limit_ns);
  tc_fence_after();
  if (__all_sync(0xffffffffu, ok)) {
    uint32_t v[4];
    tmem_ld4(tbase + (uint32_t(warp * 32) << 16), v);
    tmem_ld_wait();
#pragma unroll
    for (int c = 0; c < 4; ++c) out[(warp * 32 + lane) * 4 + c] = v[c];
  } else if (lane == 0) {
    report_status(status, MOE_ERR_TIMEOUT);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, 32);
  }
}

}  // namespace ksw

using namespace ksw;

extern "C" {

const char* moe_status_string(int status) {
  switch (status) {
    case MOE_OK: return "MOE_OK";
    case MOE_ERR_INVALID_ARG: return "MOE_ERR_INVALID_ARG";
    case MOE_ERR_UNSUPPORTED: return "MOE_ERR_UNSUPPORTED";
    case MOE_ERR_CUDA: return "MOE_ERR_CUDA";
    case MOE_ERR_TIMEOUT: return "MOE_ERR_TIMEOUT";
    case MOE_ERR_WORKSPACE: return "MOE_ERR_WORKSPACE";
    case MOE_ERR_DEVICE: return "MOE_ERR_DEVICE";
    default: return "MOE_ERR_UNKNOWN";
  }
}

const char* moe_last_error(void) { return g_last_error.c_str(); }

int moe_abi_version(void) { return MOE_B200_ABI_VERSION; }

int moe_read_status(int32_t* device_status, int32_t* host_status, int reset,
                    void* stream) {
  KSW_REQUIRE(device_status != nullptr && host_status != nullptr,
              MOE_ERR_INVALID_ARG, "moe_read_status: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  KSW_CUDA(cudaMemcpyAsync(host_status, device_status, sizeof(int32_t),
                           cudaMemcpyDeviceToHost, s));
  KSW_CUDA(cudaStreamSynchronize(s));
  if (reset) {
    KSW_CUDA(cudaMemsetAsync(device_status, 0, sizeof(int32_t), s));
    KSW_CUDA(cudaStreamSynchronize(s));
  }
  return MOE_OK;
}

int moe_selftest_wait_timeout(int32_t* device_status, int limit_us,
                              void* stream) {
  KSW_REQUIRE(device_status != nullptr, MOE_ERR_INVALID_ARG,
              "moe_selftest_wait_timeout: null status pointer");
  KSW_REQUIRE(limit_us > 0 && limit_us <= 1000000, MOE_ERR_INVALID_ARG,
              "moe_selftest_wait_timeout: limit_us must be in (0, 1e6]");
  int st = check_device(nullptr);
  if (st != MOE_OK) return st;
  selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      device_status, uint64_t(limit_us) * 1000ull);
  KSW_CUDA(cudaGetLastError());
  return MOE_OK;
}

int moe_selftest_sf_copy(const void* chunk, uint32_t* out, int32_t* device_status,
                         void* stream) {
  KSW_REQUIRE(chunk != nullptr && out != nullptr && device_status != nullptr,
              MOE_ERR_INVALID_ARG, "moe_selftest_sf_copy: null pointer");
  KSW_REQUIRE((reinterpret_cast<uintptr_t>(chunk) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(out) & 15) == 0,
              MOE_ERR_INVALID_ARG, "moe_selftest_sf_copy: buffers must be 16-byte aligned");
  int st = check_device(nullptr);
  if (st != MOE_OK) return st;
  selftest_sf_copy_kernel<<<1, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint32_t*>(chunk), out, device_status, kWaitLimitNs);
  KSW_CUDA(cudaGetLastError());
  return MOE_OK;
}

}  // extern "C"
