// gn_noalloc.cu — GroupNorm entry point that allocates nothing.
//
// sdg_groupnorm needs device scratch for its statistics, one (mean, rstd)
// pair of floats per (image, group), i.e. B * groups * 8 bytes, and expects
// the caller to pass it. Some callers have no way to
// allocate device memory: a Kotlin/JNI or other foreign-language front end
// that reaches this library only through its C ABI and links no CUDA runtime
// of its own, or a host process whose device memory is owned by another
// component's pool. For them, sdg_groupnorm_noalloc takes its scratch from a
// fixed array compiled into this library instead.
//
// The array lives in every GPU that loads the library until the process
// exits. Its device address is looked up once per device (cudaGetSymbolAddress
// with that device current) on the first call made on that device; a host
// reference to the array's name is only a host-side stand-in and is never
// handed to a kernel.
#include <mutex>
#include <string>

#include "../../include/sdg.h"
#include "sdg_kernels.h"

namespace sdg {
int op_fail(int code, const std::string& msg);
}

namespace {

// 64 KiB: GroupNorm keeps one (mean, rstd) pair per (image, group), so this
// covers batch * groups <= 8192 (e.g. 256 images at 32 groups).
constexpr size_t kNoAllocScratchBytes = size_t(64) << 10;

static __device__ __align__(256) unsigned char g_gn_scratch[kNoAllocScratchBytes];

std::mutex g_mu;
void* g_scratch_dev[64] = {nullptr};

// Device address of g_gn_scratch on the current device (looked up once per device).
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return sdg::op_fail(SDG_ERR_CUDA, std::string("groupnorm_noalloc: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return sdg::op_fail(SDG_ERR_UNSUPPORTED, "groupnorm_noalloc: device index >= 64");
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch_dev[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_gn_scratch);
    if (e != cudaSuccess || p == nullptr)
      return sdg::op_fail(SDG_ERR_CUDA, std::string("groupnorm_noalloc: cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    g_scratch_dev[dev] = p;
  }
  *out = g_scratch_dev[dev];
  return SDG_OK;
}

}  // namespace

extern "C" {

SDG_API size_t sdg_groupnorm_noalloc_max_scratch_bytes(void) { return kNoAllocScratchBytes; }

SDG_API int sdg_groupnorm_noalloc(const uint16_t* x, const uint16_t* x2, int B, int HW, int C1, int C2, int groups,
                                  const float* gamma, const float* beta, float eps, int silu, uint16_t* y,
                                  void* stream) {
  if (!x || !y || !gamma || !beta || (x2 == nullptr) != (C2 == 0) || B <= 0 || HW <= 0 || C1 <= 0 || C2 < 0 ||
      groups <= 0)
    return sdg::op_fail(SDG_ERR_ARG, "groupnorm_noalloc: bad arguments");
  const size_t need = sdg::groupnorm_scratch_bytes(B, HW, C1 + C2, groups);
  if (need > kNoAllocScratchBytes)
    return sdg::op_fail(SDG_ERR_SHAPE, "groupnorm_noalloc: shape needs " + std::to_string(need) +
                                           " bytes of scratch, more than the fixed " +
                                           std::to_string(kNoAllocScratchBytes) + "; use sdg_groupnorm");
  void* scratch = nullptr;
  int st = scratch_address(&scratch);
  if (st) return st;
  // The statistics kernel writes every (mean, rstd) pair before the apply
  // kernel reads it, so the previous call's contents need no clearing.
  sdg::GroupNormArgs a;
  a.x0 = reinterpret_cast<const __half*>(x);
  a.x1 = reinterpret_cast<const __half*>(x2);
  a.C0 = C1; a.C1 = C2; a.B = B; a.HW = HW; a.groups = groups;
  a.gamma = gamma; a.beta = beta; a.eps = eps; a.silu = silu;
  a.y = reinterpret_cast<__half*>(y);
  a.stats = static_cast<float*>(scratch);
  cudaError_t e = sdg::launch_groupnorm(a, static_cast<cudaStream_t>(stream));
  if (e == cudaErrorInvalidValue) return sdg::op_fail(SDG_ERR_SHAPE, "groupnorm_noalloc: unsupported shape");
  if (e != cudaSuccess) return sdg::op_fail(SDG_ERR_CUDA, std::string("groupnorm_noalloc: ") + cudaGetErrorString(e));
  return SDG_OK;
}

}  // extern "C"
