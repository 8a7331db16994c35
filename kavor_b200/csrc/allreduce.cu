// Tensor-parallel all-reduce over NVLink peer memory, fused with the residual
// add + RMSNorm that follows every row-parallel projection in Qwen3
// (linear.py:156-160 all_reduce -> layernorm.py:114-140 add+RMSNorm, and the
// embedding all-reduce embed_head.py:39-41 -> input_layernorm, qwen3.py:155-156).
//
// Every rank owns one "symmetric" allocation (same layout on all ranks) that
// its peers map with CUDA IPC:
//   [flags]   uint32 [2 phases][kMaxBlocks][kMaxRanks]   written by peers
//   [data 0..2] three partial-sum buffers (the row-parallel GEMM writes its
//             rank-local output straight into one of them)
//   [result]  out rows + residual rows of the two-shot exchange
// plus a private per-block counter array. A call:
//   1. block b takes v = ++counter[b] and stores v into flags[0][b][rank] of
//      every rank (st.release.sys), then waits (bounded) until its own
//      flags[0][b][p] == v for every p (ld.acquire.sys): all ranks' partials
//      are complete (they were written by earlier kernels of their streams);
//   2. one-shot (small T*H): every rank reduces every row: the N partials are
//      summed in rank order in fp32 (identical on all ranks), rounded to bf16
//      like the reference's all-reduce result, added to the residual in fp32,
//      the residual stored as bf16 and the row RMS-normalised with the
//      reference's double rounding;
//      two-shot (large T*H): rank r reduces + normalises only rows
//      t % N == r into its result buffer, a second flag round (phase 1)
//      publishes them, then every rank copies the other ranks' rows.
// Counters live in device memory, so the values advance on every CUDA-graph
// replay. Buffer reuse is safe without a trailing barrier: a rank can only
// rewrite a buffer after passing a later call's barrier, which every peer
// enters after finishing its reads of that buffer (the caller alternates data
// buffers so consecutive calls never share one).
// No TMA and no multicast are used: plain 16-byte loads/stores over NVLink.
#include "common.cuh"
#include "../../include/kavor_b200.h"

KVB_DEFINE_ERROR_WORD(allreduce)

namespace kvb {
namespace {

constexpr int kMaxRanks = 8;
constexpr int kMaxBlocks = 256;
constexpr int kThreads = 256;
constexpr int kMaxChunks = 8;  // hidden <= 256 threads x 8 chunks x 8 = 16384
constexpr int kNumData = 3;
constexpr size_t kFlagBytes = 2ull * kMaxBlocks * kMaxRanks * sizeof(uint32_t);

struct Comm {
  int rank = 0, world = 1, device = 0;
  size_t data_bytes = 0;   // capacity of one data buffer (bytes)
  uint8_t* base = nullptr;  // local symmetric allocation
  uint8_t* peer[kMaxRanks] = {};
  uint32_t* counters = nullptr;
  bool opened[kMaxRanks] = {};
};

struct Layout {
  size_t flags, data[kNumData], result, total;
};

inline Layout layout_of(size_t data_bytes) {
  Layout L;
  size_t off = 0;
  L.flags = off;
  off += (kFlagBytes + 255) & ~size_t(255);
  for (int i = 0; i < kNumData; ++i) {
    L.data[i] = off;
    off += (data_bytes + 255) & ~size_t(255);
  }
  L.result = off;
  off += 2 * ((data_bytes + 255) & ~size_t(255));
  L.total = off;
  return L;
}

struct ArArgs {
  const bf16* data[kMaxRanks];   // every rank's partial buffer for this call
  bf16* result[kMaxRanks];        // every rank's result area (two-shot)
  uint32_t* flags[kMaxRanks];     // every rank's flag area
  uint32_t* counters;             // this rank's private counters
  const bf16* residual_in;        // NULL: first layer (residual := reduced sum)
  bf16* residual_out;
  bf16* out;
  const bf16* weight;
  int rank, world, tokens, hidden, two_shot;
  size_t result_stride;           // elements between the out rows and residual rows of a result area
  float eps;
};

struct alignas(16) Vec8 {
  __nv_bfloat162 h[4];
};

__device__ __forceinline__ void st_release(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Flag round: returns false if a peer did not arrive within the spin budget.
__device__ bool flag_round(const ArArgs& a, int phase, uint32_t v, int* ok_s) {
  const int b = blockIdx.x;
  if (threadIdx.x < a.world) {
    __threadfence_system();
    st_release(a.flags[threadIdx.x] + ((size_t)phase * kMaxBlocks + b) * kMaxRanks + a.rank, v);
  }
  if (threadIdx.x == 0) *ok_s = 1;
  __syncthreads();
  if (threadIdx.x < a.world) {
    const uint32_t* f = a.flags[a.rank] + ((size_t)phase * kMaxBlocks + b) * kMaxRanks + threadIdx.x;
    if (ld_acquire(f) != v) {
      const long long t0 = clock64();
      while (ld_acquire(f) != v) {
        if (clock64() - t0 > kSpinCycles) {
          atomicOr(&g_err_allreduce, (unsigned)kErrPeerTimeout);
          *ok_s = 0;
          break;
        }
      }
    }
  }
  __syncthreads();
  return *ok_s != 0;
}

__device__ __forceinline__ void unpack8(const Vec8& v, float* f) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 p = __bfloat1622float2(v.h[i]);
    f[2 * i] = p.x;
    f[2 * i + 1] = p.y;
  }
}
__device__ __forceinline__ Vec8 pack8(const float* f) {
  Vec8 v;
#pragma unroll
  for (int i = 0; i < 4; ++i) v.h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return v;
}

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kThreads / 32; ++i) s += red[i];
  return s;
}

// Reduce row t over all ranks, add the residual, normalise; writes the bf16
// residual and output rows to (res_dst, out_dst).
__device__ void reduce_row(const ArArgs& a, int t, bf16* out_dst, bf16* res_dst, float* red) {
  const int nch = a.hidden / 8;
  const int64_t row = (int64_t)t * a.hidden;
  float v[kMaxChunks][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxChunks; ++i) {
    const int c = threadIdx.x + i * kThreads;
    if (c < nch) {
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int p = 0; p < a.world; ++p) {
        float f[8];
        unpack8(reinterpret_cast<const Vec8*>(a.data[p] + row)[c], f);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] += f[j];
      }
      float r[8];
      if (a.residual_in) unpack8(reinterpret_cast<const Vec8*>(a.residual_in + row)[c], r);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float y = bf16_round(acc[j]);  // the all-reduce result is a bf16 tensor in the reference
        v[i][j] = a.residual_in ? y + r[j] : y;
        ss += v[i][j] * v[i][j];
      }
    }
  }
  const float rstd = rsqrtf(block_sum(ss, red) / (float)a.hidden + a.eps);
  const Vec8* w = reinterpret_cast<const Vec8*>(a.weight);
#pragma unroll
  for (int i = 0; i < kMaxChunks; ++i) {
    const int c = threadIdx.x + i * kThreads;
    if (c < nch) {
      float wf[8], y[8];
      unpack8(w[c], wf);
      reinterpret_cast<Vec8*>(res_dst)[c] = pack8(v[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) y[j] = bf16_round(v[i][j] * rstd) * wf[j];
      reinterpret_cast<Vec8*>(out_dst)[c] = pack8(y);
    }
  }
}

__global__ void __launch_bounds__(kThreads) ar_add_rmsnorm_kernel(const __grid_constant__ ArArgs a) {
  __shared__ float red[kThreads / 32];
  __shared__ uint32_t v_s;
  __shared__ int ok_s;
  if (threadIdx.x == 0) {
    v_s = a.counters[blockIdx.x] + 1;
    a.counters[blockIdx.x] = v_s;
  }
  __syncthreads();
  const uint32_t v = v_s;
  if (!flag_round(a, 0, v, &ok_s)) return;
  const int nb = gridDim.x;
  if (!a.two_shot) {
    for (int t = blockIdx.x; t < a.tokens; t += nb)
      reduce_row(a, t, a.out + (int64_t)t * a.hidden, a.residual_out + (int64_t)t * a.hidden, red);
    return;
  }
  // two-shot: rows t with t % world == rank are reduced here and published
  bf16* mine = a.result[a.rank];
  for (int t = blockIdx.x; t < a.tokens; t += nb) {
    if (t % a.world != a.rank) continue;
    bf16* o = mine + (int64_t)t * a.hidden;
    reduce_row(a, t, o, o + a.result_stride, red);
    __syncthreads();
  }
  if (!flag_round(a, 1, v, &ok_s)) return;
  const int nch = a.hidden / 8;
  for (int t = blockIdx.x; t < a.tokens; t += nb) {
    const bf16* src = a.result[t % a.world] + (int64_t)t * a.hidden;
    const Vec8* so = reinterpret_cast<const Vec8*>(src);
    const Vec8* sr = reinterpret_cast<const Vec8*>(src + a.result_stride);
    Vec8* doo = reinterpret_cast<Vec8*>(a.out + (int64_t)t * a.hidden);
    Vec8* dr = reinterpret_cast<Vec8*>(a.residual_out + (int64_t)t * a.hidden);
    for (int c = threadIdx.x; c < nch; c += kThreads) {
      doo[c] = so[c];
      dr[c] = sr[c];
    }
  }
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace kvb

using namespace kvb;

extern "C" int kvb_comm_create(int rank, int world, size_t max_bytes, void** comm, void* ipc_handle) {
  if (!comm || !ipc_handle || world < 1 || world > kMaxRanks || rank < 0 || rank >= world || max_bytes == 0)
    return set_error(kInvalid, "kvb_comm_create: bad arguments (world must be 1..8)");
  Comm* c = new Comm();
  c->rank = rank;
  c->world = world;
  c->data_bytes = max_bytes;
  cudaError_t e = cudaGetDevice(&c->device);
  if (e != cudaSuccess) {
    delete c;
    return cuda_status(e, "kvb_comm_create: cudaGetDevice");
  }
  const Layout L = layout_of(max_bytes);
  e = cudaMalloc(&c->base, L.total);
  if (e == cudaSuccess) e = cudaMemset(c->base, 0, kFlagBytes);
  if (e == cudaSuccess) e = cudaMalloc(&c->counters, kMaxBlocks * sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaMemset(c->counters, 0, kMaxBlocks * sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t*>(ipc_handle), c->base);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    if (c->base) cudaFree(c->base);
    if (c->counters) cudaFree(c->counters);
    delete c;
    return cuda_status(e, "kvb_comm_create");
  }
  c->peer[rank] = c->base;
  *comm = c;
  return kOk;
}

extern "C" int kvb_comm_ipc_handle_size(void) { return (int)sizeof(cudaIpcMemHandle_t); }

extern "C" int kvb_comm_open_peers(void* comm, const void* handles) {
  Comm* c = static_cast<Comm*>(comm);
  if (!c || !handles) return set_error(kInvalid, "kvb_comm_open_peers: NULL argument");
  const cudaIpcMemHandle_t* h = static_cast<const cudaIpcMemHandle_t*>(handles);
  for (int p = 0; p < c->world; ++p) {
    if (p == c->rank || c->opened[p]) continue;
    void* ptr = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&ptr, h[p], cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_status(e, "kvb_comm_open_peers: cudaIpcOpenMemHandle");
    c->peer[p] = static_cast<uint8_t*>(ptr);
    c->opened[p] = true;
  }
  return kOk;
}

extern "C" int kvb_comm_data_buffer(void* comm, int index, void** ptr, size_t* bytes) {
  Comm* c = static_cast<Comm*>(comm);
  if (!c || !ptr || index < 0 || index >= kNumData) return set_error(kInvalid, "kvb_comm_data_buffer: bad arguments");
  *ptr = c->base + layout_of(c->data_bytes).data[index];
  if (bytes) *bytes = c->data_bytes;
  return kOk;
}

extern "C" int kvb_comm_destroy(void* comm) {
  Comm* c = static_cast<Comm*>(comm);
  if (!c) return kOk;
  int rc = kOk;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) rc = cuda_status(e, "kvb_comm_destroy: synchronize");
  for (int p = 0; p < c->world; ++p)
    if (c->opened[p]) cudaIpcCloseMemHandle(c->peer[p]);
  cudaFree(c->base);
  cudaFree(c->counters);
  delete c;
  return rc;
}

extern "C" int kvb_allreduce_add_rmsnorm(void* comm, int data_index, const void* residual_in, void* residual_out,
                                         void* out, const void* weight, int tokens, int hidden, float eps,
                                         int mode, void* stream) {
  Comm* c = static_cast<Comm*>(comm);
  if (!c || data_index < 0 || data_index >= kNumData || tokens < 0 || hidden <= 0 || mode < 0 || mode > 2)
    return set_error(kInvalid, "kvb_allreduce_add_rmsnorm: bad arguments");
  if (tokens == 0) return kOk;
  if (!residual_out || !out || !weight) return set_error(kInvalid, "kvb_allreduce_add_rmsnorm: NULL pointer");
  if (hidden % 8 || hidden > kThreads * kMaxChunks * 8 || !aligned16(out) || !aligned16(residual_out) ||
      !aligned16(weight) || (residual_in && !aligned16(residual_in)))
    return set_error(kInvalid, "kvb_allreduce_add_rmsnorm: rows must be 16-byte aligned, hidden <= 16384");
  const size_t bytes = (size_t)tokens * hidden * 2;
  if (bytes > c->data_bytes) return set_error(kInvalid, "kvb_allreduce_add_rmsnorm: %zu bytes exceed the %zu-byte buffers", bytes, c->data_bytes);
  for (int p = 0; p < c->world; ++p)
    if (!c->peer[p]) return set_error(kInvalid, "kvb_allreduce_add_rmsnorm: peer %d not opened", p);
  const Layout L = layout_of(c->data_bytes);
  ArArgs a;
  for (int p = 0; p < kMaxRanks; ++p) {
    const bool v = p < c->world;
    a.data[p] = v ? reinterpret_cast<const bf16*>(c->peer[p] + L.data[data_index]) : nullptr;
    a.result[p] = v ? reinterpret_cast<bf16*>(c->peer[p] + L.result) : nullptr;
    a.flags[p] = v ? reinterpret_cast<uint32_t*>(c->peer[p] + L.flags) : nullptr;
  }
  a.counters = c->counters;
  a.residual_in = (const bf16*)residual_in;
  a.residual_out = (bf16*)residual_out;
  a.out = (bf16*)out;
  a.weight = (const bf16*)weight;
  a.rank = c->rank;
  a.world = c->world;
  a.tokens = tokens;
  a.hidden = hidden;
  // mode 0: automatic (one-shot up to 512 KiB per rank), 1: one-shot, 2: two-shot
  a.two_shot = c->world > 1 && (mode == 2 || (mode == 0 && bytes > (512u << 10)));
  a.result_stride = ((c->data_bytes + 255) & ~size_t(255)) / 2;
  a.eps = eps;
  const int blocks = tokens < kMaxBlocks ? tokens : kMaxBlocks;
  ar_add_rmsnorm_kernel<<<blocks, kThreads, 0, (cudaStream_t)stream>>>(a);
  return cuda_status(cudaGetLastError(), "kvb_allreduce_add_rmsnorm launch");
}
