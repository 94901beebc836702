// abi.cu -- C-ABI plumbing: error state, device error word, environment
// switches, TMA tensor-map encoding, and the elementwise / normalisation glue
// entry points (rmsnorm, vector_add, swiglu_f16, embedding_f16).
#include <cuda_runtime.h>

#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <tuple>

#include "common.cuh"
#include "kernels.cuh"

namespace b200 {

namespace {
thread_local std::string g_last_error;
std::mutex g_mu;

// One word per device that loads the library: kernels OR error bits into it
// instead of hanging when a bounded wait runs out.
__device__ unsigned int g_device_error;
}  // namespace

int set_error(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int set_cuda_error(cudaError_t err, const char* what) {
  g_last_error = std::string(cudaGetErrorName(err)) + ": " + cudaGetErrorString(err) +
                 " (in " + what + ")";
  return ENGINE_ERR_CUDA;
}

bool always_sync_check() {
  static const bool v = [] {
    const char* e = std::getenv("ENGINE_ALWAYS_SYNC_CHECK");
    return e != nullptr && e[0] != '\0' && e[0] != '0';
  }();
  return v;
}

bool pdl_enabled() {
  static const bool v = [] {
    const char* e = std::getenv("ENGINE_PDL");
    return !(e != nullptr && e[0] == '0');
  }();
  return v;
}

unsigned long long wait_limit_ns() {
  static const unsigned long long v = [] {
    const char* e = std::getenv("ENGINE_WAIT_TIMEOUT_MS");
    long ms = e ? std::strtol(e, nullptr, 10) : 0;
    if (ms <= 0) ms = 2000;
    return static_cast<unsigned long long>(ms) * 1000000ull;
  }();
  return v;
}

namespace {
struct DevInfo {
  int sms = 0;
  int smem_optin = 0;
  unsigned int* err = nullptr;
};
std::map<int, DevInfo> g_dev;

DevInfo& dev_info() {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(g_mu);
  DevInfo& d = g_dev[dev];
  if (d.sms == 0) {
    cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&d.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) == cudaSuccess) {
      d.err = static_cast<unsigned int*>(p);
    }
    if (d.sms <= 0) d.sms = 148;
  }
  return d;
}
}  // namespace

int sm_count() { return dev_info().sms; }
int max_smem_optin() { return dev_info().smem_optin; }
unsigned int* device_error_word() { return dev_info().err; }

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, what);
  if (always_sync_check()) {
    e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return set_cuda_error(e, what);
    unsigned int flags = 0;
    e = cudaMemcpyFromSymbol(&flags, g_device_error, sizeof(flags));
    if (e != cudaSuccess) return set_cuda_error(e, what);
    if (flags != 0) {
      const unsigned int zero = 0;
      cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero));
      return set_error(ENGINE_ERR_DEVICE, std::string(what) + ": device error flags " +
                                              std::to_string(flags));
    }
  }
  return ENGINE_OK;
}

EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      return static_cast<EncodeTiledFn>(nullptr);
    }
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

namespace {
using TmapKey = std::tuple<int, const void*, int, uint64_t, uint64_t, uint64_t, uint32_t, uint32_t>;
std::map<TmapKey, CUtensorMap> g_tmaps;
}  // namespace

// L2 sector promotion of the 2-D tensor maps (CUtensorMapL2promotion: 0 none,
// 1 64B, 2 128B, 3 256B), a compile-time tunable.
#ifndef ENGINE_TMAP_L2_PROMOTION
#define ENGINE_TMAP_L2_PROMOTION 3
#endif

bool make_tmap_2d(CUtensorMap* out, const void* ptr, CUtensorMapDataType dtype, int elem_bytes,
                  uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows,
                  uint32_t box_cols) {
  int dev = 0;
  cudaGetDevice(&dev);
  const TmapKey key{dev, ptr, static_cast<int>(dtype), rows, cols, ld, box_rows, box_cols};
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_tmaps.find(key);
    if (it != g_tmaps.end()) {
      *out = it->second;
      return true;
    }
  }
  EncodeTiledFn enc = encode_tiled_fn();
  if (enc == nullptr) {
    set_error(ENGINE_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
    return false;
  }
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {ld * static_cast<uint64_t>(elem_bytes)};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUtensorMap m;
  std::memset(&m, 0, sizeof(m));
  const CUresult r = enc(&m, dtype, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         static_cast<CUtensorMapL2promotion>(ENGINE_TMAP_L2_PROMOTION),
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error(ENGINE_ERR_UNSUPPORTED,
              "cuTensorMapEncodeTiled failed (code " + std::to_string(static_cast<int>(r)) +
                  "): pointer/stride not 16-byte aligned or box too large");
    return false;
  }
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_tmaps.size() > 4096) g_tmaps.clear();  // bound the cache
    g_tmaps.emplace(key, m);
  }
  *out = m;
  return true;
}

bool make_tmap_3d(CUtensorMap* out, const void* ptr, CUtensorMapDataType dtype, int elem_bytes,
                  const uint64_t (&dims)[3], const uint64_t (&strides)[2],
                  const uint32_t (&box)[3]) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (enc == nullptr) {
    set_error(ENGINE_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
    return false;
  }
  const cuuint64_t d[3] = {dims[0], dims[1], dims[2]};
  const cuuint64_t st[2] = {strides[0] * static_cast<uint64_t>(elem_bytes),
                            strides[1] * static_cast<uint64_t>(elem_bytes)};
  const cuuint32_t b[3] = {box[0], box[1], box[2]};
  const cuuint32_t estr[3] = {1, 1, 1};
  std::memset(out, 0, sizeof(*out));
  const CUresult r = enc(out, dtype, 3, const_cast<void*>(ptr), d, st, b, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error(ENGINE_ERR_UNSUPPORTED,
              "cuTensorMapEncodeTiled (3-D) failed (code " + std::to_string(static_cast<int>(r)) +
                  "): pointer/stride not 16-byte aligned or box too large");
    return false;
  }
  return true;
}

namespace {
std::map<int, cudaMemPool_t> g_pools;
}  // namespace

void* scratch_alloc(size_t bytes, cudaStream_t stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  cudaMemPool_t pool = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_pools.find(dev);
    if (it == g_pools.end()) {
      cudaMemPoolProps props = {};
      props.allocType = cudaMemAllocationTypePinned;
      props.handleTypes = cudaMemHandleTypeNone;
      props.location.type = cudaMemLocationTypeDevice;
      props.location.id = dev;
      cudaError_t e = cudaMemPoolCreate(&pool, &props);
      if (e != cudaSuccess) {
        set_cuda_error(e, "cudaMemPoolCreate (scratch)");
        return nullptr;
      }
      uint64_t keep = ~0ull;  // keep freed blocks cached in the pool
      cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
      g_pools.emplace(dev, pool);
    } else {
      pool = it->second;
    }
  }
  void* p = nullptr;
  cudaError_t e = cudaMallocFromPoolAsync(&p, bytes, pool, stream);
  if (e != cudaSuccess) {
    set_cuda_error(e, "cudaMallocFromPoolAsync (scratch)");
    return nullptr;
  }
  return p;
}

void scratch_free(void* p, cudaStream_t stream) {
  if (p != nullptr) cudaFreeAsync(p, stream);
}

// ---------------------------------------------------------------- kernels

namespace {

// One block per row (grid-stride over rows).  Squares are summed in double and
// the scale is formed as float(1 / sqrt(mean + eps)) in double, the reference's
// arithmetic (src/cpu_ref/rmsnorm_cpu.cpp:19-43); out = (x * scale) * w in float.
// RES: the row is first s = x + residual in float, written to sum_out and
// normalised in place of x (src/cpu_ref/residual_rmsnorm_cpu.cpp:19-51).  Each
// thread reads back in the second pass only the sum_out elements it wrote.
template <bool RES>
__global__ void __launch_bounds__(256) rmsnorm_f32_kernel(const float* __restrict__ in,
                                                          const float* __restrict__ res,
                                                          const float* __restrict__ w,
                                                          float* __restrict__ out,
                                                          float* __restrict__ sum_out,
                                                          int64_t rows, int64_t cols,
                                                          float eps) {
  __shared__ double s_part[8];
  __shared__ float s_scale;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* src = in + r * cols;
    const float* rsrc = RES ? res + r * cols : nullptr;
    float* ssum = RES ? sum_out + r * cols : nullptr;
    double ss = 0.0;
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
      float x = src[c];
      if constexpr (RES) {
        x = __fadd_rn(x, rsrc[c]);
        ssum[c] = x;
      }
      const double v = static_cast<double>(x);
      ss = __dadd_rn(ss, __dmul_rn(v, v));
    }
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
      double t = 0.0;
      for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) t += s_part[i];
      s_scale = static_cast<float>(1.0 / sqrt(t / static_cast<double>(cols) +
                                              static_cast<double>(eps)));
    }
    __syncthreads();
    const float scale = s_scale;
    float* dst = out + r * cols;
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
      const float wv = w ? w[c] : 1.0f;
      dst[c] = __fmul_rn(__fmul_rn(RES ? ssum[c] : src[c], scale), wv);
    }
    __syncthreads();
  }
}

__global__ void vector_add_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                  float* __restrict__ out, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    out[i] = __fadd_rn(a[i], b[i]);
  }
}

// silu(g) * u in float with the library expf; FP16 out (round to nearest even).
__global__ void swiglu_f16_kernel(const __half* __restrict__ g, const __half* __restrict__ u,
                                  __half* __restrict__ out, int64_t n) {
  pdl_trigger();
  pdl_wait();
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    out[i] = swiglu_h(g[i], u[i]);
  }
}

__global__ void embedding_f16_kernel(const __half* __restrict__ table,
                                     const int32_t* __restrict__ ids, __half* __restrict__ out,
                                     int64_t hidden, int64_t vocab, unsigned int* err) {
  pdl_trigger();
  pdl_wait();
  const int64_t t = blockIdx.x;
  const int32_t id = ids[t];
  const bool ok = id >= 0 && id < vocab;
  if (!ok && threadIdx.x == 0 && err) atomicOr(err, kErrBadArgument);
  const __half* src = table + static_cast<int64_t>(ok ? id : 0) * hidden;
  __half* dst = out + t * hidden;
  for (int64_t c = threadIdx.x; c < hidden; c += blockDim.x) {
    dst[c] = ok ? src[c] : __float2half_rn(0.0f);
  }
}

int grid_for(int64_t n, int threads) {
  const int64_t want = (n + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
  return static_cast<int>(want < cap ? (want > 0 ? want : 1) : cap);
}

}  // namespace
}  // namespace b200

using namespace b200;

extern "C" {

int engine_abi_version(void) { return 1; }

const char* engine_last_error(void) { return b200::g_last_error.c_str(); }

int engine_device_status(int device, unsigned int* flags) {
  B200_ENTRY_BEGIN
  B200_REQUIRE(flags != nullptr, "engine_device_status: flags is null");
  int prev = 0;
  B200_CUDA(cudaGetDevice(&prev));
  B200_CUDA(cudaSetDevice(device));
  cudaError_t e = cudaDeviceSynchronize();
  unsigned int v = 0;
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v));
  if (e == cudaSuccess) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero));
  }
  // A kernel that gave up may have left a stream-K tile half counted.
  if (e == cudaSuccess && v != 0) {
    sk_workspace_reset(device);
    e = cudaDeviceSynchronize();
  }
  cudaSetDevice(prev);
  if (e != cudaSuccess) return set_cuda_error(e, "engine_device_status");
  *flags = v;
  return ENGINE_OK;
  B200_ENTRY_END
}

int engine_cuda_rmsnorm(const float* in, const float* weight, float* out, int64_t rows,
                        int64_t cols, float eps, engine_stream_t stream) {
  B200_ENTRY_BEGIN
  B200_REQUIRE(rows >= 0 && cols >= 0, "rmsnorm: negative dimension");
  B200_REQUIRE(in != nullptr && out != nullptr, "rmsnorm: null device pointer");
  B200_REQUIRE(eps >= 0.0f, "rmsnorm: eps must be non-negative");
  if (rows == 0 || cols == 0) return ENGINE_OK;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 32;
  const int grid = static_cast<int>(rows < cap ? rows : cap);
  rmsnorm_f32_kernel<false><<<grid, 256, 0, stream>>>(in, nullptr, weight, out, nullptr, rows,
                                                       cols, eps);
  return check_launch("rmsnorm");
  B200_ENTRY_END
}

int engine_cuda_residual_rmsnorm(const float* x, const float* residual, const float* weight,
                                 float* norm_out, float* sum_out, int64_t rows, int64_t cols,
                                 float eps, engine_stream_t stream) {
  B200_ENTRY_BEGIN
  B200_REQUIRE(rows >= 0 && cols >= 0, "residual_rmsnorm: negative dimension");
  B200_REQUIRE(x != nullptr && residual != nullptr && norm_out != nullptr && sum_out != nullptr,
               "residual_rmsnorm: null device pointer");
  B200_REQUIRE(eps >= 0.0f, "residual_rmsnorm: eps must be non-negative");
  if (rows == 0 || cols == 0) return ENGINE_OK;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 32;
  const int grid = static_cast<int>(rows < cap ? rows : cap);
  rmsnorm_f32_kernel<true><<<grid, 256, 0, stream>>>(x, residual, weight, norm_out, sum_out, rows,
                                                      cols, eps);
  return check_launch("residual_rmsnorm");
  B200_ENTRY_END
}

int engine_cuda_vector_add(const float* a, const float* b, float* out, int64_t n,
                           engine_stream_t stream) {
  B200_ENTRY_BEGIN
  B200_REQUIRE(a != nullptr, "vector_add: a is null");
  B200_REQUIRE(b != nullptr, "vector_add: b is null");
  B200_REQUIRE(out != nullptr, "vector_add: out is null");
  B200_REQUIRE(n >= 0, "vector_add: n must be non-negative");
  if (n == 0) return ENGINE_OK;
  vector_add_kernel<<<grid_for(n, 256), 256, 0, stream>>>(a, b, out, n);
  return check_launch("vector_add");
  B200_ENTRY_END
}

int engine_cuda_swiglu_f16(const engine_half_t* gate, const engine_half_t* up,
                           engine_half_t* out, int64_t n, engine_stream_t stream) {
  B200_ENTRY_BEGIN
  B200_REQUIRE(gate != nullptr, "swiglu_fp16: gate is null");
  B200_REQUIRE(up != nullptr, "swiglu_fp16: up is null");
  B200_REQUIRE(out != nullptr, "swiglu_fp16: out is null");
  B200_REQUIRE(n >= 0, "swiglu_fp16: n must be non-negative");
  if (n == 0) return ENGINE_OK;
  B200_CUDA(launch_pdl(swiglu_f16_kernel, dim3(grid_for(n, 256)), dim3(256), 0, stream,
                       reinterpret_cast<const __half*>(gate), reinterpret_cast<const __half*>(up),
                       reinterpret_cast<__half*>(out), n));
  return check_launch("swiglu_fp16");
  B200_ENTRY_END
}

int engine_cuda_embedding_f16(const engine_half_t* table, const int32_t* ids,
                              engine_half_t* out, int64_t num_tokens, int64_t hidden,
                              int64_t vocab, engine_stream_t stream) {
  B200_ENTRY_BEGIN
  B200_REQUIRE(table != nullptr && ids != nullptr && out != nullptr,
               "embedding_fp16: null device pointer");
  B200_REQUIRE(num_tokens >= 0, "embedding_fp16: num_tokens must be non-negative");
  B200_REQUIRE(hidden >= 0, "embedding_fp16: hidden_dim must be non-negative");
  B200_REQUIRE(vocab > 0, "embedding_fp16: vocab_size must be positive");
  if (num_tokens == 0 || hidden == 0) return ENGINE_OK;
  B200_REQUIRE(num_tokens <= 0x7fffffff, "embedding_fp16: too many tokens");
  B200_CUDA(launch_pdl(embedding_f16_kernel, dim3(static_cast<unsigned>(num_tokens)), dim3(256), 0,
                       stream, reinterpret_cast<const __half*>(table), ids,
                       reinterpret_cast<__half*>(out), hidden, vocab, device_error_word()));
  return check_launch("embedding_fp16");
  B200_ENTRY_END
}

}  // extern "C"
