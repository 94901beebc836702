// tp_comm.cu -- tensor-parallel communicator over NVLink peer memory, and the
// row-split projection fused with its all-reduce.
//
// One process per GPU.  Each rank allocates one device region:
//
//   recv   [2 parities][world sources][cap]  u64  {payload, call number} words:
//          the payload is one FP32 partial (fused projection) or two FP16
//          partials (all-reduce of an FP16 tensor)
//   epoch  [kTpCtas]                         u32  this rank's call count, per CTA
//
// The ranks exchange the regions' CUDA IPC handles through the host (the
// Python layer uses torch.distributed) and map every peer's region.
//
// A call is one-shot and push-based, in the low-latency form of NCCL's LL
// protocol: every partial value travels as ONE 64-bit word that carries its
// own validity (high half = the call number).
// 1. CTA b computes its share of this rank's partial result (for the fused
//    projection: GEMV row blocks of X W_r^T) and stores each value, tagged,
//    into slot [parity][rank] of EVERY rank's recv area.  These are plain
//    64-bit system-scope stores over NVLink.  There is no fence, no flag and
//    no barrier.
// 2. CTA b then reads, for each of its elements, the `world` words of slots
//    [parity][0..world) of its own recv area.  It re-reads each word until its
//    tag equals the call number; the wait is bounded by the library's limit.
//    It adds the values in rank order 0..world-1, adds the residual, rounds
//    once to FP16 and writes Y.
// An aligned 64-bit access is single-copy atomic, so a word with the right tag
// holds the right value.  Every rank adds the same values in the same order,
// so all ranks hold bit-identical results, which the replicated residual
// stream needs.  The reference has no multi-GPU code; this replaces an NCCL
// all-reduce (sum, FP16) after the O and down projections.
//
// Ordering rules:
// - Every call launches the same grid of kTpCtas CTAs (all co-resident; the
//   communicator checks occupancy), so per-CTA call counts agree and the
//   parity (count & 1) is the same in every CTA of a call.
// - A rank can be at most one call ahead of another: it finishes call k only
//   after every peer's words for k have arrived, and a peer writes them in its
//   own call k, which starts after its call k-1 has finished.  Two parities
//   therefore keep a fast rank's words for call k+1 away from the words a slow
//   rank is still reading for call k.
// - All calls on one communicator must be stream-ordered on each rank.
// - Counts live in device memory, so a captured CUDA graph replays correctly.
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>
#include <new>

#include "common.cuh"
#include "gemv_core.cuh"
#include "kernels.cuh"

struct engine_tp_comm {
  int rank = 0;
  int world = 1;
  int device = 0;
  int64_t cap = 0;                 // words per (parity, source) slot
  uint8_t* region = nullptr;       // this rank's region
  size_t recv_bytes = 0, epoch_off = 0, region_bytes = 0;
  cudaIpcMemHandle_t handle;
  uint8_t* peer[b200::kTpMaxWorld] = {};
  bool ipc_opened[b200::kTpMaxWorld] = {};
  bool ready = false;
  __half* partial = nullptr;       // scratch for the unfused (GEMM) path: cap halves
};

namespace b200 {
namespace {

struct TpArgs {
  unsigned long long* recv[kTpMaxWorld];  // rank s's recv area as mapped on this GPU
  unsigned long long* own;                // recv[rank] (read with a static index)
  uint32_t* epoch;                        // this rank's per-CTA call counts
  int rank, world;
  int64_t cap;
  unsigned int* err;
  unsigned long long limit_ns;
};

/// Thread 0 advances this CTA's call count; returns it to every thread.
__device__ __forceinline__ uint32_t tp_begin(const TpArgs& a, uint32_t* s_e) {
  if (threadIdx.x == 0) {
    const uint32_t e = a.epoch[blockIdx.x] + 1u;
    a.epoch[blockIdx.x] = e;
    *s_e = e;
  }
  __syncthreads();
  return *s_e;
}

__device__ __forceinline__ unsigned long long* tp_slot(const TpArgs& a, int dst, uint32_t e,
                                                       int src) {
  return a.recv[dst] + (static_cast<int64_t>(e & 1u) * a.world + src) * a.cap;
}

/// Stores 32 payload bits for word idx, tagged with call e, into every rank's slot.
__device__ __forceinline__ void tp_push_bits(const TpArgs& a, uint32_t e, int64_t idx,
                                             uint32_t bits) {
  const unsigned long long w = (static_cast<unsigned long long>(e) << 32) | bits;
#pragma unroll
  for (int s = 0; s < kTpMaxWorld; ++s) {  // static indices keep the pointers in registers
    if (s < a.world) {
      asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(tp_slot(a, s, e, a.rank) + idx),
                   "l"(w)
                   : "memory");
    }
  }
}

/// Stores FP32 value v of element idx, tagged with call e, into every rank's slot.
__device__ __forceinline__ void tp_push(const TpArgs& a, uint32_t e, int64_t idx, float v) {
  tp_push_bits(a, e, idx, __float_as_uint(v));
}

/// Reads word idx of call e from source s's slot (re-reading until its tag is
/// e; bounded by the wait limit).  Returns false on a time-out.
__device__ __forceinline__ bool tp_wait_word(const TpArgs& a, const unsigned long long* p,
                                             uint32_t e, uint32_t& bits,
                                             unsigned long long& t0) {
  unsigned long long w;
  int spins = 0;
  while (true) {
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    if (static_cast<uint32_t>(w >> 32) == e) break;
    if ((++spins & 63) == 0) {
      const unsigned long long now = globaltimer();
      if (t0 == 0) t0 = now;
      if (now - t0 > a.limit_ns) {
        if (a.err) atomicOr(a.err, kErrWaitTimeout);
        return false;
      }
    }
  }
  bits = static_cast<uint32_t>(w);
  return true;
}

/// Sums over sources 0..world-1 (in that order) of the half2 word idx of call e.
__device__ __forceinline__ bool tp_gather_h2(const TpArgs& a, uint32_t e, int64_t idx, float& v0,
                                             float& v1, unsigned long long& t0) {
  const unsigned long long* base = a.own + static_cast<int64_t>(e & 1u) * a.world * a.cap + idx;
  float s0 = 0.0f, s1 = 0.0f;
  for (int s = 0; s < a.world; ++s) {
    uint32_t bits;
    if (!tp_wait_word(a, base + s * a.cap, e, bits, t0)) return false;
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&bits));
    s0 += f.x;
    s1 += f.y;
  }
  v0 = s0;
  v1 = s1;
  return true;
}

/// Sum over sources 0..world-1 (in that order) of element idx of call e.  Each
/// word is re-read until its tag is e; gives up after the wait limit (sets the
/// device error word, returns false).
__device__ __forceinline__ bool tp_gather(const TpArgs& a, uint32_t e, int64_t idx, float& sum,
                                          unsigned long long& t0) {
  const unsigned long long* base = a.own + static_cast<int64_t>(e & 1u) * a.world * a.cap + idx;
  float v = 0.0f;
  for (int s = 0; s < a.world; ++s) {
    uint32_t bits;
    if (!tp_wait_word(a, base + s * a.cap, e, bits, t0)) return false;
    v += __uint_as_float(bits);
  }
  sum = v;
  return true;
}

// Fused row-split projection + all-reduce for M <= 4 activation rows:
// Y[m, n] = sum_s (X_s W_s^T)[m, n] + R[m, n] on every rank.  Row blocks of W
// (kNkVecWarps / SK groups x RPW rows) are dealt to the kTpCtas CTAs
// round-robin; phase 1 is the decode GEMV (nk_block_dots).  Launched as a
// programmatic dependent: the first weight chunks are prefetched into L2 while
// the preceding kernel drains.
template <int MR, int RPW, int SK, int U>
__global__ void __launch_bounds__(kNkVecWarps * 32, 2)
    tp_linear_ar_kernel(const TpArgs a, const __half* __restrict__ W,
                        const __half* __restrict__ X, const __half* __restrict__ R,
                        __half* __restrict__ Y, int64_t N, int64_t K) {
  constexpr int GROUPS = kNkVecWarps / SK;
  constexpr int ROWS = GROUPS * RPW;
  __shared__ float red[kNkVecWarps][MR * RPW];
  __shared__ uint32_t s_e;
  const int64_t nblocks = (N + ROWS - 1) / ROWS;
  pdl_trigger();
  if (blockIdx.x < nblocks) nk_block_prefetch<RPW, SK, U>(W, N, K, blockIdx.x);
  pdl_wait();
  const uint32_t e = tp_begin(a, &s_e);
  for (int64_t b = blockIdx.x; b < nblocks; b += gridDim.x) {
    nk_block_dots<MR, RPW, SK, U, false>(W, X, nullptr, N, K, b, red);
    for (int o = threadIdx.x; o < GROUPS * MR * RPW; o += blockDim.x) {
      const int g = o / (MR * RPW);
      const int rem = o % (MR * RPW);
      const int m = rem / RPW;
      const int r = rem % RPW;
      const int64_t row = (b * GROUPS + g) * RPW + r;
      if (row >= N) continue;
      float v = 0.0f;
#pragma unroll
      for (int q = 0; q < SK; ++q) v += red[g * SK + q][m * RPW + r];
      tp_push(a, e, m * N + row, v);
    }
    __syncthreads();  // `red` is reused by the next block
  }
  unsigned long long t0 = 0;
  for (int64_t b = blockIdx.x; b < nblocks; b += gridDim.x) {
    for (int o = threadIdx.x; o < MR * ROWS; o += blockDim.x) {
      const int m = o / ROWS;
      const int64_t row = b * ROWS + o % ROWS;
      if (row >= N) continue;
      const int64_t idx = m * N + row;
      float v;
      if (!tp_gather(a, e, idx, v, t0)) return;
      if (R != nullptr) v += __half2float(R[idx]);
      Y[idx] = __float2half_rn(v);
    }
  }
}

// All-reduce of an FP16 partial P[n] (any producer): Y = sum_s P_s + R.  The
// values already are FP16, so each tagged word carries TWO of them (a half2 in
// the low half): half the NVLink bytes of FP32 words, the same sums.  CTA b
// owns element pairs [b*per, (b+1)*per).
__global__ void __launch_bounds__(256, 2)
    tp_allreduce_kernel(const TpArgs a, const __half* __restrict__ P,
                        const __half* __restrict__ R, __half* __restrict__ Y, int64_t n,
                        int64_t per) {
  __shared__ uint32_t s_e;
  pdl_trigger();
  pdl_wait();
  const uint32_t e = tp_begin(a, &s_e);
  const int64_t npairs = (n + 1) / 2;
  const int64_t lo = static_cast<int64_t>(blockIdx.x) * per;
  const int64_t hi = (lo + per < npairs) ? lo + per : npairs;
  for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    const __half x0 = P[2 * i];
    const __half x1 = (2 * i + 1 < n) ? P[2 * i + 1] : __float2half_rn(0.0f);
    const __half2 h = __halves2half2(x0, x1);
    tp_push_bits(a, e, i, *reinterpret_cast<const uint32_t*>(&h));
  }
  unsigned long long t0 = 0;
  for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    float v0 = 0.0f, v1 = 0.0f;
    if (!tp_gather_h2(a, e, i, v0, v1, t0)) return;
    if (R != nullptr) v0 += __half2float(R[2 * i]);
    Y[2 * i] = __float2half_rn(v0);
    if (2 * i + 1 < n) {
      if (R != nullptr) v1 += __half2float(R[2 * i + 1]);
      Y[2 * i + 1] = __float2half_rn(v1);
    }
  }
}

size_t align256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

TpArgs make_args(const engine_tp_comm* c) {
  TpArgs a;
  std::memset(&a, 0, sizeof(a));
  for (int s = 0; s < c->world; ++s) a.recv[s] = reinterpret_cast<unsigned long long*>(c->peer[s]);
  a.own = a.recv[c->rank];
  a.epoch = reinterpret_cast<uint32_t*>(c->region + c->epoch_off);
  a.rank = c->rank;
  a.world = c->world;
  a.cap = c->cap;
  a.err = device_error_word();
  a.limit_ns = wait_limit_ns();
  return a;
}

template <typename Kern>
bool fits_co_resident(Kern k, int threads) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, threads, 0) != cudaSuccess)
    return false;
  return per_sm * sm_count() >= kTpCtas;
}

int check_comm(const engine_tp_comm* c) {
  if (c == nullptr) return set_error(ENGINE_ERR_INVALID, "tp: comm is null");
  if (!c->ready) return set_error(ENGINE_ERR_INVALID, "tp: comm is not open (call engine_tp_comm_open)");
  int dev = -1;
  B200_CUDA(cudaGetDevice(&dev));
  if (dev != c->device)
    return set_error(ENGINE_ERR_INVALID, "tp: the current device is not the communicator's device");
  return ENGINE_OK;
}

int launch_allreduce(const engine_tp_comm* c, const __half* P, const __half* R, __half* Y,
                     int64_t n, cudaStream_t stream) {
  const int64_t per = ((n + 1) / 2 + kTpCtas - 1) / kTpCtas;  // element pairs per CTA
  B200_CUDA(launch_pdl(tp_allreduce_kernel, dim3(kTpCtas), dim3(256), 0, stream, make_args(c), P,
                       R, Y, n, per));
  return check_launch("tp_allreduce_f16");
}

// One warp group per RPW weight rows, SK = 1 (each warp streams whole rows):
// 16 rows per CTA for M <= 2 (N = 4096 is one row block per CTA), 8 for M > 2
// (register budget of the 2-CTA/SM launch).
template <int MR>
struct TpGemvCfg {
  static constexpr int RPW = (MR <= 2) ? 2 : 1;
  static constexpr int SK = 1;
  static constexpr int U = (MR == 1) ? 4 : 2;
};

template <int MR>
int launch_linear_ar(const engine_tp_comm* c, const __half* X, const __half* W, const __half* R,
                     __half* Y, int64_t N, int64_t K, cudaStream_t stream) {
  using C = TpGemvCfg<MR>;
  B200_CUDA(launch_pdl(tp_linear_ar_kernel<MR, C::RPW, C::SK, C::U>, dim3(kTpCtas),
                       dim3(kNkVecWarps * 32), 0, stream, make_args(c), W, X, R, Y, N, K));
  return check_launch("tp_linear_allreduce_f16");
}

template <int MR>
bool linear_ar_fits() {
  using C = TpGemvCfg<MR>;
  return fits_co_resident(tp_linear_ar_kernel<MR, C::RPW, C::SK, C::U>, kNkVecWarps * 32);
}

bool kernels_fit() {
  return fits_co_resident(tp_allreduce_kernel, 256) && linear_ar_fits<1>() &&
         linear_ar_fits<2>() && linear_ar_fits<3>() && linear_ar_fits<4>();
}

}  // namespace
}  // namespace b200

using namespace b200;

extern "C" {

int engine_tp_comm_create(int rank, int world, int64_t max_elems, engine_tp_comm_t** comm) {
  B200_ENTRY_BEGIN
  B200_REQUIRE(comm != nullptr, "tp_comm_create: comm is null");
  *comm = nullptr;
  B200_REQUIRE(world >= 1 && world <= kTpMaxWorld, "tp_comm_create: world must be in [1, 8]");
  B200_REQUIRE(rank >= 0 && rank < world, "tp_comm_create: rank must be in [0, world)");
  B200_REQUIRE(max_elems > 0, "tp_comm_create: max_elems must be positive");
  // 2 parities x world x cap 8-byte words: bounded so the region size cannot overflow.
  B200_REQUIRE(max_elems <= (int64_t(1) << 28), "tp_comm_create: max_elems must be at most 2^28");
  if (!kernels_fit())
    return set_error(ENGINE_ERR_UNSUPPORTED,
                     "tp_comm_create: the communicator kernels cannot keep 256 CTAs co-resident");
  int device = 0;
  B200_CUDA(cudaGetDevice(&device));
  auto* c = new (std::nothrow) engine_tp_comm();
  if (c == nullptr) return set_error(ENGINE_ERR_INTERNAL, "tp_comm_create: out of host memory");
  c->rank = rank;
  c->world = world;
  c->cap = (max_elems + 31) / 32 * 32;
  c->device = device;
  c->recv_bytes = align256(static_cast<size_t>(2) * world * c->cap * sizeof(unsigned long long));
  c->epoch_off = c->recv_bytes;
  c->region_bytes = c->epoch_off + align256(static_cast<size_t>(kTpCtas) * 4);
  cudaError_t e = cudaMalloc(&c->region, c->region_bytes);
  if (e == cudaSuccess) e = cudaMemset(c->region, 0, c->region_bytes);
  if (e == cudaSuccess) e = cudaMalloc(&c->partial, static_cast<size_t>(c->cap) * sizeof(__half));
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&c->handle, c->region);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    if (c->region) cudaFree(c->region);
    if (c->partial) cudaFree(c->partial);
    delete c;
    return set_cuda_error(e, "tp_comm_create");
  }
  c->peer[rank] = c->region;
  *comm = c;
  return ENGINE_OK;
  B200_ENTRY_END
}

int engine_tp_comm_handle(const engine_tp_comm_t* comm, void* handle) {
  B200_ENTRY_BEGIN
  B200_REQUIRE(comm != nullptr && handle != nullptr, "tp_comm_handle: null pointer");
  static_assert(sizeof(cudaIpcMemHandle_t) == ENGINE_TP_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &comm->handle, ENGINE_TP_HANDLE_BYTES);
  return ENGINE_OK;
  B200_ENTRY_END
}

int engine_tp_comm_open(engine_tp_comm_t* comm, const void* handles) {
  B200_ENTRY_BEGIN
  B200_REQUIRE(comm != nullptr && handles != nullptr, "tp_comm_open: null pointer");
  B200_REQUIRE(!comm->ready, "tp_comm_open: already open");
  const auto* h = static_cast<const uint8_t*>(handles);
  B200_REQUIRE(std::memcmp(h + comm->rank * ENGINE_TP_HANDLE_BYTES, &comm->handle,
                           ENGINE_TP_HANDLE_BYTES) == 0,
               "tp_comm_open: handles[rank] is not this rank's handle");
  for (int s = 0; s < comm->world; ++s) {
    if (s == comm->rank) continue;
    const uint8_t* hs = h + s * ENGINE_TP_HANDLE_BYTES;
    if (std::memcmp(hs, &comm->handle, ENGINE_TP_HANDLE_BYTES) == 0) {
      comm->peer[s] = comm->region;  // loopback: the same region (single-process tests)
      continue;
    }
    cudaIpcMemHandle_t ih;
    std::memcpy(&ih, hs, ENGINE_TP_HANDLE_BYTES);
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, ih, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int q = 0; q < s; ++q) {
        if (comm->ipc_opened[q]) cudaIpcCloseMemHandle(comm->peer[q]);
        comm->ipc_opened[q] = false;
        if (q != comm->rank) comm->peer[q] = nullptr;
      }
      return set_cuda_error(e, "tp_comm_open (cudaIpcOpenMemHandle)");
    }
    comm->peer[s] = static_cast<uint8_t*>(p);
    comm->ipc_opened[s] = true;
  }
  comm->ready = true;
  return ENGINE_OK;
  B200_ENTRY_END
}

int engine_tp_comm_destroy(engine_tp_comm_t* comm) {
  B200_ENTRY_BEGIN
  if (comm == nullptr) return ENGINE_OK;
  for (int s = 0; s < comm->world; ++s) {
    if (comm->ipc_opened[s]) cudaIpcCloseMemHandle(comm->peer[s]);
  }
  if (comm->region) cudaFree(comm->region);
  if (comm->partial) cudaFree(comm->partial);
  delete comm;
  return ENGINE_OK;
  B200_ENTRY_END
}

int engine_tp_allreduce_f16(engine_tp_comm_t* comm, const engine_half_t* partial,
                            const engine_half_t* residual, engine_half_t* y, int64_t n,
                            engine_stream_t stream) {
  B200_ENTRY_BEGIN
  const int rc = check_comm(comm);
  if (rc != ENGINE_OK) return rc;
  B200_REQUIRE(n >= 0, "tp_allreduce_f16: n must be non-negative");
  B200_REQUIRE(partial != nullptr && y != nullptr, "tp_allreduce_f16: null device pointer");
  B200_REQUIRE(n <= comm->cap, "tp_allreduce_f16: n exceeds the communicator's max_elems");
  // n == 0 still runs the exchange: every rank must make the same calls.
  return launch_allreduce(comm, reinterpret_cast<const __half*>(partial),
                          reinterpret_cast<const __half*>(residual), reinterpret_cast<__half*>(y), n,
                          static_cast<cudaStream_t>(stream));
  B200_ENTRY_END
}

int engine_tp_linear_allreduce_f16(engine_tp_comm_t* comm, const engine_half_t* X,
                                   const engine_half_t* W, const engine_half_t* residual,
                                   engine_half_t* Y, int64_t M, int64_t N, int64_t K,
                                   engine_stream_t stream) {
  B200_ENTRY_BEGIN
  const int rc = check_comm(comm);
  if (rc != ENGINE_OK) return rc;
  B200_REQUIRE(M >= 0 && N >= 0 && K >= 0, "tp_linear_allreduce_f16: negative dimension");
  B200_REQUIRE(X != nullptr && W != nullptr && Y != nullptr,
               "tp_linear_allreduce_f16: null device pointer");
  B200_REQUIRE(N == 0 || M <= comm->cap / N,
               "tp_linear_allreduce_f16: M*N exceeds the communicator's max_elems");
  auto st = static_cast<cudaStream_t>(stream);
  const auto* x = reinterpret_cast<const __half*>(X);
  const auto* w = reinterpret_cast<const __half*>(W);
  const auto* r = reinterpret_cast<const __half*>(residual);
  auto* y = reinterpret_cast<__half*>(Y);
  const bool vec = K > 0 && (K % 8 == 0) && (reinterpret_cast<uintptr_t>(W) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(X) % 16 == 0);
  if (vec && M >= 1 && M <= 4) {
    switch (M) {
      case 1: return launch_linear_ar<1>(comm, x, w, r, y, N, K, st);
      case 2: return launch_linear_ar<2>(comm, x, w, r, y, N, K, st);
      case 3: return launch_linear_ar<3>(comm, x, w, r, y, N, K, st);
      default: return launch_linear_ar<4>(comm, x, w, r, y, N, K, st);
    }
  }
  // Larger batches: the tensor-core projection into the communicator's scratch,
  // then the one-shot all-reduce (two launches, same stream).
  const int rc2 = engine_cuda_linear_f16(X, W, nullptr,
                                         reinterpret_cast<engine_half_t*>(comm->partial), M, N, K,
                                         stream);
  if (rc2 != ENGINE_OK) return rc2;
  return launch_allreduce(comm, comm->partial, r, y, M * N, st);
  B200_ENTRY_END
}

}  // extern "C"
