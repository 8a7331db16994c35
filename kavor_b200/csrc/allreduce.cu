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
constexpr size_t kMcFlagBytes = 2ull * kMaxBlocks * sizeof(uint32_t);  // switch-reduced arrival counters

struct Comm {
  int rank = 0, world = 1, device = 0;
  size_t data_bytes = 0;   // capacity of one data buffer (bytes)
  uint8_t* base = nullptr;  // local symmetric allocation
  uint8_t* peer[kMaxRanks] = {};
  uint8_t* mc = nullptr;    // NVLink multicast mapping of the area (NULL: none)
  uint32_t* counters = nullptr;     // [kMaxBlocks] calls per block (peer flag rounds)
  uint32_t* mc_counters = nullptr;  // [2][kMaxBlocks] calls per block that ran the first / second switch arrival
  bool opened[kMaxRanks] = {};
  bool owns_area = true;    // false: the area was attached (allocated and mapped by the caller)
  int max_blocks = kMaxBlocks;  // grid cap of a call (kvb_comm_set_max_blocks)
};

struct Layout {
  size_t flags, mc_flags, data[kNumData], result, total;
};

inline Layout layout_of(size_t data_bytes) {
  Layout L;
  size_t off = 0;
  L.flags = off;
  off += (kFlagBytes + 255) & ~size_t(255);
  L.mc_flags = off;
  off += (kMcFlagBytes + 255) & ~size_t(255);
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
  uint32_t* mc_counters;          // this rank's private counters: [phase][block] switch rounds run
  uint32_t* mc_flags;             // multicast address of the arrival counters (NVLS modes)
  uint32_t* local_mc_flags;       // this rank's copy of them
  int skip_out_copy, skip_res_copy;  // NVLS two-shot: out / residual_out are this rank's result rows
  const bf16* residual_in;        // NULL: first layer (residual := reduced sum)
  bf16* residual_out;
  bf16* out;
  const bf16* weight;
  const bf16* mc_data;            // multicast address of this call's partial buffer (NVLS modes)
  bf16* mc_result;                // multicast address of the result area (NVLS two-shot)
  int rank, world, tokens, hidden, two_shot, nvls;
  size_t result_stride;           // elements between the out rows and residual rows of a result area
  float eps;
};

struct alignas(16) Vec8 {
  __nv_bfloat162 h[4];
};

// NVLink SHARP: one 16-byte load that returns the sum over every rank's copy
// (reduced in the switch, fp32 accumulation, one bf16 rounding), and one
// 16-byte store that lands in every rank's copy.
__device__ __forceinline__ Vec8 mc_ld_reduce(const bf16* mc) {
  Vec8 v;
  uint32_t* r = reinterpret_cast<uint32_t*>(&v);
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "l"(mc)
               : "memory");
  return v;
}
__device__ __forceinline__ void mc_store(bf16* mc, const Vec8& v) {
  const uint32_t* r = reinterpret_cast<const uint32_t*>(&v);
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc), "r"(r[0]), "r"(r[1]),
               "r"(r[2]), "r"(r[3])
               : "memory");
}

__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Flag round: block b tells every rank "my part of call v is ready" and waits
// until every rank told it the same. Returns false if a peer did not arrive
// within the spin budget. `publish` = this kernel wrote the data the peers
// will read (two-shot results): a system-scope release fence orders the
// block's writes (all threads, via the preceding __syncthreads) before the
// flag. The partial sums of the first round were written by earlier kernels,
// which completed before this one started, so that round needs no fence.
template <int W>
__device__ bool flag_round(const ArArgs& a, int phase, uint32_t v, bool publish, int* ok_s) {
  const int b = blockIdx.x;
  if (threadIdx.x < W) {
    if (publish) asm volatile("fence.acq_rel.sys;" ::: "memory");
    st_relaxed_sys(a.flags[threadIdx.x] + ((size_t)phase * kMaxBlocks + b) * kMaxRanks + a.rank, v);
  }
  if (threadIdx.x == 0) *ok_s = 1;
  __syncthreads();
  if (threadIdx.x < W) {
    const uint32_t* f = a.flags[a.rank] + ((size_t)phase * kMaxBlocks + b) * kMaxRanks + threadIdx.x;
    // flags only grow (each is the peer's call count), so "at least v" also
    // holds when a fast peer has already moved on to its next call
    if ((int)(ld_acquire(f) - v) < 0) {
      const long long t0 = clock64();
      while ((int)(ld_acquire(f) - v) < 0) {
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

// Switch flag round: thread 0 adds 1 to block b's arrival counter on every
// rank at once (multimem.red through the NVSwitch) and waits until its own
// copy reaches W x (calls of this block so far). `publish`: a system-scope
// release fence first orders the block's multicast stores before the arrival.
__device__ bool mc_round(const ArArgs& a, int phase, uint32_t target, bool publish, int* ok_s) {
  __syncthreads();
  if (threadIdx.x == 0) {
    *ok_s = 1;
    uint32_t* mc = a.mc_flags + (size_t)phase * kMaxBlocks + blockIdx.x;
    if (publish) asm volatile("fence.acq_rel.sys;" ::: "memory");
    asm volatile("multimem.red.relaxed.sys.global.add.u32 [%0], %1;" ::"l"(mc), "r"(1u) : "memory");
    const uint32_t* f = a.local_mc_flags + (size_t)phase * kMaxBlocks + blockIdx.x;
    if ((int)(ld_acquire(f) - target) < 0) {
      const long long t0 = clock64();
      while ((int)(ld_acquire(f) - target) < 0) {
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

// Reduce row t over the W ranks, add the residual, normalise; writes the bf16
// residual and output rows to (res_dst, out_dst). Thread j owns the 16-byte
// chunks j, j + 256, ... (NCH of them); the loads of G chunks x W ranks (8
// vectors) are all issued before any is used, so a row costs one NVLink round
// trip per group instead of one per (chunk, rank). MC: the sum comes from the
// switch (one multicast load per chunk); ST_MC: the rows are stored through the
// multicast mapping into every rank's result area.
template <int W, int NCH, bool MC, bool ST_MC>
__device__ void reduce_row(const ArArgs& a, int t, bf16* out_dst, bf16* res_dst, float* red) {
  constexpr int WL = MC ? 1 : W;  // vectors loaded per chunk
  constexpr int G = (8 / WL) < NCH ? (8 / WL) : NCH;
  const int nch = a.hidden / 8;
  const int64_t row = (int64_t)t * a.hidden;
  float v[NCH][8];
  float ss = 0.f;
#pragma unroll
  for (int g0 = 0; g0 < NCH; g0 += G) {
    Vec8 in[G][WL];
    Vec8 rin[G];
#pragma unroll
    for (int i = 0; i < G; ++i) {
      const int c = threadIdx.x + (g0 + i) * kThreads;
      if (g0 + i < NCH && c < nch) {
        if constexpr (MC) {
          in[i][0] = mc_ld_reduce(a.mc_data + row + (int64_t)c * 8);
        } else {
#pragma unroll
          for (int p = 0; p < W; ++p) in[i][p] = reinterpret_cast<const Vec8*>(a.data[p] + row)[c];
        }
        if (a.residual_in) rin[i] = reinterpret_cast<const Vec8*>(a.residual_in + row)[c];
      }
    }
#pragma unroll
    for (int i = 0; i < G; ++i) {
      const int c = threadIdx.x + (g0 + i) * kThreads;
      if (g0 + i < NCH && c < nch) {
        float acc[8], f[8];
        unpack8(in[i][0], acc);
#pragma unroll
        for (int p = 1; p < WL; ++p) {  // rank order: identical sums on every rank
          unpack8(in[i][p], f);
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[j] += f[j];
        }
        float r[8];
        if (a.residual_in) unpack8(rin[i], r);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float y = bf16_round(acc[j]);  // the all-reduce result is a bf16 tensor in the reference
          v[g0 + i][j] = a.residual_in ? y + r[j] : y;
          ss += v[g0 + i][j] * v[g0 + i][j];
        }
      }
    }
  }
  const float rstd = rsqrtf(block_sum(ss, red) / (float)a.hidden + a.eps);
  const Vec8* w = reinterpret_cast<const Vec8*>(a.weight);
#pragma unroll
  for (int i = 0; i < NCH; ++i) {
    const int c = threadIdx.x + i * kThreads;
    if (c < nch) {
      float wf[8], y[8];
      unpack8(w[c], wf);
#pragma unroll
      for (int j = 0; j < 8; ++j) y[j] = bf16_round(v[i][j] * rstd) * wf[j];
      if constexpr (ST_MC) {
        mc_store(res_dst + (int64_t)c * 8, pack8(v[i]));
        mc_store(out_dst + (int64_t)c * 8, pack8(y));
      } else {
        reinterpret_cast<Vec8*>(res_dst)[c] = pack8(v[i]);
        reinterpret_cast<Vec8*>(out_dst)[c] = pack8(y);
      }
    }
  }
}

// Rows t = blockIdx.x, blockIdx.x + gridDim.x, ... of the two-shot result
// area `src` (out rows, then residual rows `result_stride` further) -> out,
// residual_out.
template <int NCH>
__device__ void copy_rows(const ArArgs& a, int t, const bf16* src) {
  const int nch = a.hidden / 8;
  const Vec8* so = reinterpret_cast<const Vec8*>(src);
  const Vec8* sr = reinterpret_cast<const Vec8*>(src + a.result_stride);
  Vec8* doo = reinterpret_cast<Vec8*>(a.out + (int64_t)t * a.hidden);
  Vec8* dr = reinterpret_cast<Vec8*>(a.residual_out + (int64_t)t * a.hidden);
  Vec8 bo[NCH], br[NCH];
#pragma unroll
  for (int i = 0; i < NCH; ++i) {
    const int c = threadIdx.x + i * kThreads;
    if (c < nch) {
      bo[i] = so[c];
      br[i] = sr[c];
    }
  }
#pragma unroll
  for (int i = 0; i < NCH; ++i) {
    const int c = threadIdx.x + i * kThreads;
    if (c < nch) {
      if (!a.skip_out_copy) doo[c] = bo[i];
      if (!a.skip_res_copy) dr[c] = br[i];
    }
  }
}

// Two blocks per SM at most 128 registers: every block of a call (<= 256) is
// resident at once, so no block can wait on a peer block that is not running.
template <int W, int NCH>
__global__ void __launch_bounds__(kThreads, 2) ar_add_rmsnorm_kernel(const __grid_constant__ ArArgs a) {
  kernel_entry();
  __shared__ float red[kThreads / 32];
  __shared__ uint32_t v_s;
  __shared__ int ok_s;
  __shared__ uint32_t v1_s;
  if (threadIdx.x == 0) {
    // each flag word counts its own rounds: the switch round-1 word only
    // advances in two-shot calls, so it gets a counter of its own
    uint32_t* ctr = a.nvls ? a.mc_counters : a.counters;
    v_s = ctr[blockIdx.x] + 1;
    ctr[blockIdx.x] = v_s;
    if (a.nvls == 2) {
      v1_s = a.mc_counters[kMaxBlocks + blockIdx.x] + 1;
      a.mc_counters[kMaxBlocks + blockIdx.x] = v1_s;
    }
  }
  __syncthreads();
  const uint32_t v = v_s;
  const int nb = gridDim.x;
  const int64_t H = a.hidden;
  if (a.nvls) {
    const uint32_t target = (uint32_t)W * v;  // round-0 word: W per switch call of this block
    if (!mc_round(a, 0, target, false, &ok_s)) return;
    if (a.nvls == 1) {  // every rank reduces every row through the switch
      for (int t = blockIdx.x; t < a.tokens; t += nb)
        reduce_row<W, NCH, true, false>(a, t, a.out + t * H, a.residual_out + t * H, red);
      return;
    }
    // two-shot: block b of rank r reduces rows (b + k nb) W + r through the
    // switch and multicasts out + residual rows into every rank's result area
    for (int g = blockIdx.x; g * W < a.tokens; g += nb) {
      const int t = g * W + a.rank;
      if (t >= a.tokens) continue;
      bf16* o = a.mc_result + t * H;
      reduce_row<W, NCH, true, true>(a, t, o, o + a.result_stride, red);
    }
    if (!mc_round(a, 1, (uint32_t)W * v1_s, true, &ok_s)) return;  // round-1 word: W per two-shot call
    if (a.skip_out_copy && a.skip_res_copy) return;  // the caller reads the result rows in place
    for (int g = blockIdx.x; g * W < a.tokens; g += nb)
      for (int p = 0; p < W; ++p) {
        const int t = g * W + p;
        if (t < a.tokens) copy_rows<NCH>(a, t, a.result[a.rank] + t * H);
      }
    return;
  }
  if (!flag_round<W>(a, 0, v, false, &ok_s)) return;
  if (!a.two_shot) {
    for (int t = blockIdx.x; t < a.tokens; t += nb)
      reduce_row<W, NCH, false, false>(a, t, a.out + t * H, a.residual_out + t * H, red);
    return;
  }
  // two-shot over peer memory: rows t with t % W == rank are reduced here and
  // published, then every rank copies every row from its owner
  bf16* mine = a.result[a.rank];
  for (int t = blockIdx.x; t < a.tokens; t += nb) {
    if (t % W != a.rank) continue;
    bf16* o = mine + t * H;
    reduce_row<W, NCH, false, false>(a, t, o, o + a.result_stride, red);
  }
  __syncthreads();
  if (!flag_round<W>(a, 1, v, true, &ok_s)) return;
  for (int t = blockIdx.x; t < a.tokens; t += nb) copy_rows<NCH>(a, t, a.result[t % W] + t * H);
}

template <int W>
cudaError_t launch_w(const ArArgs& a, int blocks, int nch, cudaStream_t st) {
  const int per = (nch + kThreads - 1) / kThreads;
  if (per <= 1) return launch_kernel(ar_add_rmsnorm_kernel<W, 1>, dim3(blocks), dim3(kThreads), 0, st, a);
  if (per <= 2) return launch_kernel(ar_add_rmsnorm_kernel<W, 2>, dim3(blocks), dim3(kThreads), 0, st, a);
  if (per <= 4) return launch_kernel(ar_add_rmsnorm_kernel<W, 4>, dim3(blocks), dim3(kThreads), 0, st, a);
  return launch_kernel(ar_add_rmsnorm_kernel<W, 8>, dim3(blocks), dim3(kThreads), 0, st, a);
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Which exchange a call uses (mode 0 = automatic): peer two-shot when the
// one-shot would read more than 8 MiB per rank; with a multicast mapping and
// more than two ranks the switch modes instead, two-shot from 8 rows per rank.
void choose_mode(int world, bool multicast, int tokens, int hidden, int mode, int* two_shot, int* nvls) {
  const size_t bytes = (size_t)tokens * hidden * 2;
  *two_shot = world > 2 && (mode == 2 || (mode == 0 && bytes * world > (8u << 20)));
  if (mode == 2 && world > 1) *two_shot = 1;
  *nvls = 0;
  if (mode == 3 || mode == 4) *nvls = mode - 2;
  if (mode == 0 && multicast && world > 2) *nvls = (size_t)tokens >= (size_t)world * 8 ? 2 : 1;
}

}  // namespace
}  // namespace kvb

using namespace kvb;

extern "C" int kvb_comm_create(int rank, int world, size_t max_bytes, void** comm, void* ipc_handle) {
  if (!comm || !ipc_handle || rank < 0 || rank >= world || max_bytes == 0)
    return set_error(kInvalid, "kvb_comm_create: bad arguments");
  if (world != 1 && world != 2 && world != 4 && world != 8)
    return set_error(kUnsupported, "kvb_comm_create: world size must be 1, 2, 4 or 8 (got %d)", world);
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
  if (e == cudaSuccess) e = cudaMalloc(&c->counters, 3 * kMaxBlocks * sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaMemset(c->counters, 0, 3 * kMaxBlocks * sizeof(uint32_t));
  if (e == cudaSuccess) c->mc_counters = c->counters + kMaxBlocks;
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
  if (c->owns_area) cudaFree(c->base);
  cudaFree(c->counters);
  delete c;
  return rc;
}

extern "C" int kvb_comm_area_size(size_t max_bytes, size_t* bytes) {
  if (!bytes || max_bytes == 0) return set_error(kInvalid, "kvb_comm_area_size: bad arguments");
  *bytes = layout_of(max_bytes).total;
  return kOk;
}

extern "C" int kvb_comm_attach(int rank, int world, const uint64_t* peer_bases, uint64_t multicast_base,
                               size_t area_bytes, size_t max_bytes, void** comm) {
  if (!comm || !peer_bases || rank < 0 || rank >= world || max_bytes == 0)
    return set_error(kInvalid, "kvb_comm_attach: bad arguments");
  if (world != 1 && world != 2 && world != 4 && world != 8)
    return set_error(kUnsupported, "kvb_comm_attach: world size must be 1, 2, 4 or 8 (got %d)", world);
  const Layout L = layout_of(max_bytes);
  if (area_bytes < L.total)
    return set_error(kInvalid, "kvb_comm_attach: area of %zu bytes, %zu needed", area_bytes, L.total);
  for (int p = 0; p < world; ++p)
    if (!peer_bases[p] || (peer_bases[p] & 255)) return set_error(kInvalid, "kvb_comm_attach: peer %d base NULL or unaligned", p);
  if (multicast_base & 255) return set_error(kInvalid, "kvb_comm_attach: multicast base unaligned");
  Comm* c = new Comm();
  c->rank = rank;
  c->world = world;
  c->data_bytes = max_bytes;
  c->owns_area = false;
  c->base = reinterpret_cast<uint8_t*>(peer_bases[rank]);
  for (int p = 0; p < world; ++p) c->peer[p] = reinterpret_cast<uint8_t*>(peer_bases[p]);
  c->mc = reinterpret_cast<uint8_t*>(multicast_base);
  cudaError_t e = cudaGetDevice(&c->device);
  if (e == cudaSuccess) e = cudaMalloc(&c->counters, 3 * kMaxBlocks * sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaMemset(c->counters, 0, 3 * kMaxBlocks * sizeof(uint32_t));
  if (e == cudaSuccess) c->mc_counters = c->counters + kMaxBlocks;
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    if (c->counters) cudaFree(c->counters);
    delete c;
    return cuda_status(e, "kvb_comm_attach");
  }
  *comm = c;
  return kOk;
}

extern "C" int kvb_comm_result_rows(void* comm, void** out_rows, void** residual_rows) {
  Comm* c = static_cast<Comm*>(comm);
  if (!c || !out_rows || !residual_rows) return set_error(kInvalid, "kvb_comm_result_rows: bad arguments");
  const Layout L = layout_of(c->data_bytes);
  *out_rows = c->base + L.result;
  *residual_rows = c->base + L.result + ((c->data_bytes + 255) & ~size_t(255));
  return kOk;
}

extern "C" int kvb_allreduce_plan(int world, int has_multicast, int tokens, int hidden, int mode, int* plan) {
  if (!plan || world < 1 || tokens < 0 || hidden <= 0 || mode < 0 || mode > 4)
    return set_error(kInvalid, "kvb_allreduce_plan: bad arguments");
  choose_mode(world, has_multicast != 0, tokens, hidden, mode, &plan[0], &plan[1]);
  return kOk;
}

extern "C" int kvb_comm_set_max_blocks(void* comm, int max_blocks) {
  Comm* c = static_cast<Comm*>(comm);
  if (!c || max_blocks < 1 || max_blocks > kMaxBlocks)
    return set_error(kInvalid, "kvb_comm_set_max_blocks: need a communicator and 1 <= max_blocks <= %d (got %d)",
                     kMaxBlocks, max_blocks);
  c->max_blocks = max_blocks;
  return kOk;
}

extern "C" int kvb_comm_has_multicast(void* comm) {
  Comm* c = static_cast<Comm*>(comm);
  return c && c->mc ? 1 : 0;
}

extern "C" int kvb_allreduce_add_rmsnorm(void* comm, int data_index, const void* residual_in, void* residual_out,
                                         void* out, const void* weight, int tokens, int hidden, float eps,
                                         int mode, void* stream) {
  Comm* c = static_cast<Comm*>(comm);
  if (!c || data_index < 0 || data_index >= kNumData || tokens < 0 || hidden <= 0 || mode < 0 || mode > 4)
    return set_error(kInvalid, "kvb_allreduce_add_rmsnorm: bad arguments");
  if (mode >= 3 && !c->mc)
    return set_error(kUnsupported, "kvb_allreduce_add_rmsnorm: mode %d needs an NVLink multicast mapping", mode);
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
  a.mc_counters = c->mc_counters;
  a.mc_flags = c->mc ? reinterpret_cast<uint32_t*>(c->mc + L.mc_flags) : nullptr;
  a.local_mc_flags = reinterpret_cast<uint32_t*>(c->base + L.mc_flags);
  a.residual_in = (const bf16*)residual_in;
  a.residual_out = (bf16*)residual_out;
  a.out = (bf16*)out;
  a.weight = (const bf16*)weight;
  a.rank = c->rank;
  a.world = c->world;
  a.tokens = tokens;
  a.hidden = hidden;
  // mode 0: automatic, 1/2: one-/two-shot over peer memory, 3/4: one-/two-shot
  // through the NVLink switch (multicast). Peer one-shot reads (world - 1)
  // full partials per rank, peer two-shot 2 (world - 1) / world of them plus a
  // second flag round; switch one-shot reads one reduced copy, switch
  // two-shot 1/world of it and multicasts 2/world back.
  choose_mode(c->world, c->mc != nullptr, tokens, hidden, mode, &a.two_shot, &a.nvls);
  a.mc_data = c->mc ? reinterpret_cast<const bf16*>(c->mc + L.data[data_index]) : nullptr;
  a.mc_result = c->mc ? reinterpret_cast<bf16*>(c->mc + L.result) : nullptr;
  a.result_stride = ((c->data_bytes + 255) & ~size_t(255)) / 2;
  a.eps = eps;
  const size_t res_off = ((c->data_bytes + 255) & ~size_t(255));
  a.skip_out_copy = out == c->base + L.result;
  a.skip_res_copy = residual_out == c->base + L.result + res_off;
  if (a.nvls != 2 && (a.skip_out_copy || a.skip_res_copy))
    return set_error(kInvalid, "kvb_allreduce_add_rmsnorm: out / residual_out in the result area need the switch two-shot mode");
  // rows per block: one row (one-shot, peer two-shot) or one group of W rows (switch two-shot)
  const int rows = a.nvls == 2 ? (tokens + c->world - 1) / c->world : tokens;
  const int blocks = rows < c->max_blocks ? rows : c->max_blocks;
  const int nch = hidden / 8;
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e;
  switch (c->world) {
    case 1: e = launch_w<1>(a, blocks, nch, st); break;
    case 2: e = launch_w<2>(a, blocks, nch, st); break;
    case 4: e = launch_w<4>(a, blocks, nch, st); break;
    default: e = launch_w<8>(a, blocks, nch, st); break;
  }
  return cuda_status(e, "kvb_allreduce_add_rmsnorm launch");
}
