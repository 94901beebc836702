// noalloc.cu -- engine_cuda_rmsnorm_linear_f16_noalloc: the small-batch fused
// RMSNorm -> linear projection for callers that cannot allocate device memory.
//
// Who needs it: a serving loop that reserves every device buffer at start-up
// and must not allocate on the request path (an allocation there can fail under
// memory pressure or wait behind other allocations, and either breaks a latency
// budget), and a host whose device memory belongs to another allocator -- a
// framework's caching allocator or a fixed arena -- that this library must not
// go around.  engine_cuda_rmsnorm_linear_f16 with 5 <= M <= 32 takes its
// normalised activations from a stream-ordered pool; this variant keeps them
// in a fixed array compiled into the library instead.
//
// The array: kNoallocScratchBytes (2 MiB) of file-scope device memory, held by
// every GPU that loads the library until the process exits.  It fits the hi/lo
// activations of up to 32 rows with K <= 16384.  Every call overwrites all the
// rows it reads (padding rows are written as zeros each time), so nothing in it
// has to start at zero and no state carries from one call to the next.  All
// calls share the one array: two calls whose work overlaps on the GPU (for
// example on two streams without ordering between them) race on it.
//
// Its device address is looked up once per device with cudaGetSymbolAddress,
// with that device current, by the first call made on that device; host code
// never hands the array's name itself to a kernel (in host code that name is
// only a host-side stand-in).  Make that first call before any stream capture.
#include <mutex>

#include "common.cuh"
#include "kernels.cuh"

namespace b200 {
namespace {

constexpr int64_t kNoallocMaxRows = 32;
constexpr int64_t kNoallocMaxK = 16384;
constexpr size_t kNoallocScratchBytes =
    static_cast<size_t>(2 * kNoallocMaxRows * kNoallocMaxK) * sizeof(__half);  // 2 MiB

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device (looked up once).
int noalloc_scratch(void** out) {
  int dev = 0;
  B200_CUDA(cudaGetDevice(&dev));
  B200_REQUIRE(dev >= 0 && dev < kMaxDevices, "rmsnorm_linear_f16_noalloc: device index too large");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return set_cuda_error(e, "cudaGetSymbolAddress(noalloc scratch)");
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return ENGINE_OK;
}

}  // namespace
}  // namespace b200

using namespace b200;

extern "C" {

int engine_cuda_rmsnorm_linear_f16_noalloc(const engine_half_t* x, const engine_half_t* gamma,
                                           const engine_half_t* W, const engine_half_t* residual,
                                           engine_half_t* Y, int64_t M, int64_t N, int64_t K,
                                           float eps, engine_stream_t stream) {
  B200_ENTRY_BEGIN
  B200_REQUIRE(M >= 0 && N >= 0 && K >= 0, "rmsnorm_linear_f16_noalloc: negative dimension");
  B200_REQUIRE(x != nullptr && W != nullptr && Y != nullptr,
               "rmsnorm_linear_f16_noalloc: null device pointer");
  B200_REQUIRE(eps >= 0.0f, "rmsnorm_linear_f16_noalloc: eps must be non-negative");
  if (M == 0 || N == 0 || K == 0) return ENGINE_OK;
  if (M > kNoallocMaxRows || K > kNoallocMaxK) {
    return set_error(ENGINE_ERR_UNSUPPORTED,
                     "rmsnorm_linear_f16_noalloc: M=" + std::to_string(M) + ", K=" +
                         std::to_string(K) + " exceeds the fixed scratch (M <= " +
                         std::to_string(kNoallocMaxRows) + ", K <= " +
                         std::to_string(kNoallocMaxK) + ")");
  }
  if (K % 8 != 0 || reinterpret_cast<uintptr_t>(W) % 16 != 0) {
    return set_error(ENGINE_ERR_UNSUPPORTED,
                     "rmsnorm_linear_f16_noalloc: K must be a multiple of 8 and W 16-byte aligned");
  }
  void* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc != ENGINE_OK) return rc;
  int hb = 8;
  while (hb < M) hb <<= 1;
  __half* x2 = static_cast<__half*>(scratch);
  rc = rmsnorm_hilo(reinterpret_cast<const __half*>(x), reinterpret_cast<const __half*>(gamma), x2,
                    M, K, hb, eps, stream);
  if (rc != ENGINE_OK) return rc;
  return gemm_tc_general(x2, W, residual, Y, M, N, K, /*bf16=*/false, /*b_kmajor=*/true,
                         /*hilo=*/true, hb, stream);
  B200_ENTRY_END
}

}  // extern "C"
