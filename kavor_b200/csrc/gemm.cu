// bf16 GEMM on the 5th-generation tensor cores: Y[M, N] = X[M, K] * W[N, K]^T
// (F.linear of linear.py:50,73,157 and embed_head.py:61), fp32 accumulation in
// TMEM, bf16 output.
//
// Orientation ("swap AB"): the UMMA A operand is a 128-row slab of the weight
// W (128 output features), the B operand is a tile of MT token rows of X, so
// the accumulator D[feature, token] lives in 128 TMEM lanes x MT columns. At
// decode batch sizes (M <= 256 tokens) one tile covers every token and the
// kernel streams each weight byte exactly once — the GEMM is HBM-bound and its
// roofline is weight bytes / HBM bandwidth. Larger M is tiled in MT = 256
// token chunks.
//
//   warp 0      TMA producer: W box {64 K, 128 rows} + X box {64 K, MT rows},
//               128-byte swizzle, into a `stages`-deep mbarrier ring;
//   warp 1      allocates TMEM, one elected thread issues
//               tcgen05.mma.cta_group::1.kind::f16 (M=128, N=MT, K=16) x4 per
//               stage and tcgen05.commit's the stage back to the producer;
//   warps 2..5  epilogue: tcgen05.ld 32x32b of their TMEM lane quarter,
//               thread = output feature, columns = tokens; coalesced bf16
//               stores (or fp32 split-K partials).
// Split-K: the K range of a weight slab is cut into `splits` parts so that
// (slabs x splits) fills the 148 SMs in whole waves; every part stores fp32
// partials to the workspace and the last CTA to finish a slab (atomic ticket)
// sums the parts in split order (deterministic) and writes bf16, then resets
// its ticket to zero for the next call.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "../../include/kavor_b200.h"

KVB_DEFINE_ERROR_WORD(gemm)

namespace kvb {
namespace {

constexpr int kBK = 64;          // K elements per stage = one 128-byte swizzle row
constexpr int kBN = 128;         // weight rows per slab = UMMA M
constexpr int kThreads = 192;    // 6 warps
constexpr int kEpiWarp0 = 2;
constexpr int kABytes = kBN * kBK * 2;  // 16 KB

struct GemmArgs {
  bf16* y;
  int64_t ldy;
  float* partial;   // [splits][m_pad][n_pad] fp32 when splits > 1
  int* tickets;     // [n_tiles * m_tiles]
  int M, N;
  int n_tiles, m_tiles, splits, kb_total, kb_per_split;
  int n_pad, m_pad;
  uint32_t idesc;
};

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}

// K-major operand tile [rows][64 bf16] with 128-byte swizzle: 8-row groups of
// 1024 B (stride byte offset), leading byte offset unused (16 B), version 1
// (sm100 descriptor), layout type 2 = SWIZZLE_128B.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(0u));
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive TMEM columns of this warp's 32 lanes -> 32 registers per thread.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

template <int MT>
struct Cfg {
  static constexpr int kBBytes = MT * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBudget = MT <= 64 ? 110 * 1024 : 200 * 1024;  // two CTAs per SM when MT <= 64
  static constexpr int kStagesRaw = kBudget / kStageBytes;
  static constexpr int kStages = kStagesRaw > 8 ? 8 : (kStagesRaw < 2 ? 2 : kStagesRaw);
  static constexpr int kTmemCols = MT < 32 ? 32 : MT;
  static constexpr int kSmem = kStages * kStageBytes + 1024;
};

template <int MT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                const __grid_constant__ GemmArgs a) {
  using C = Cfg<MT>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[C::kStages];
  __shared__ __align__(8) uint64_t empty_bar[C::kStages];
  __shared__ __align__(8) uint64_t accum_bar;
  __shared__ uint32_t tmem_base_s;
  __shared__ int last_s;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int bid = blockIdx.x;
  const int split = bid % a.splits;
  bid /= a.splits;
  const int m_tile = bid % a.m_tiles;
  const int n_tile = bid / a.m_tiles;
  const int kb0 = split * a.kb_per_split;
  const int kb1 = min(kb0 + a.kb_per_split, a.kb_total);
  const int nkb = kb1 - kb0;
  const int n0 = n_tile * kBN, m0 = m_tile * MT;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), 1);
    }
    mbar_init(smem_u32(&accum_bar), 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)),
                 "r"(C::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_d = tmem_base_s;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0 && nkb > 0) {
      prefetch_tensormap(&wmap);
      prefetch_tensormap(&xmap);
      for (int i = 0; i < nkb; ++i) {
        const int s = i % C::kStages;
        if (i >= C::kStages && !mbar_wait(smem_u32(&empty_bar[s]), ((i / C::kStages) - 1) & 1, &g_err_gemm)) break;
        const uint32_t sa = smem_u32(smem + s * C::kStageBytes);
        const uint32_t fb = smem_u32(&full_bar[s]);
        mbar_arrive_expect_tx(fb, C::kStageBytes);
        tma_load_2d(sa, &wmap, (kb0 + i) * kBK, n0, fb);
        tma_load_2d(sa + kABytes, &xmap, (kb0 + i) * kBK, m0, fb);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0 && nkb > 0) {
      bool ok = true;
      for (int i = 0; i < nkb && ok; ++i) {
        const int s = i % C::kStages;
        if (!mbar_wait(smem_u32(&full_bar[s]), (i / C::kStages) & 1, &g_err_gemm)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + s * C::kStageBytes);
        const uint64_t da = smem_desc_sw128(sa), db = smem_desc_sw128(sa + kABytes);
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k)  // +32 bytes along K inside the swizzle atom = +2 in the address field
          umma_bf16(tmem_d, da + 2 * k, db + 2 * k, a.idesc, (i > 0 || k > 0) ? 1u : 0u);
        umma_commit(smem_u32(&empty_bar[s]));
      }
      umma_commit(smem_u32(&accum_bar));
      // do not leave the CTA (and free TMEM) with MMAs in flight
      mbar_wait(smem_u32(&accum_bar), 0, &g_err_gemm);
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int n = n0 + q * 32 + lane;
    const bool ok = nkb > 0 && mbar_wait(smem_u32(&accum_bar), 0, &g_err_gemm);
    tc_fence_after();
    const uint32_t trow = tmem_d + ((uint32_t)(q * 32) << 16);
    if (a.splits == 1) {
      if (ok) {
#pragma unroll 1
        for (int c = 0; c < MT; c += (MT < 32 ? 16 : 32)) {
          float v[32];
          if constexpr (MT < 32) tmem_ld16(trow + c, v); else tmem_ld32(trow + c, v);
          if (n < a.N) {
#pragma unroll
            for (int j = 0; j < (MT < 32 ? 16 : 32); ++j) {
              const int m = m0 + c + j;
              if (m < a.M) a.y[(int64_t)m * a.ldy + n] = __float2bfloat16_rn(v[j]);
            }
          }
        }
      }
    } else {
      // fp32 partial of this split, then the last split of the slab reduces
      float* part = a.partial + ((int64_t)split * a.m_pad + m0) * a.n_pad + n;
#pragma unroll 1
      for (int c = 0; c < MT; c += (MT < 32 ? 16 : 32)) {
        float v[32];
        if (ok) {
          if constexpr (MT < 32) tmem_ld16(trow + c, v); else tmem_ld32(trow + c, v);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = 0.f;
        }
#pragma unroll
        for (int j = 0; j < (MT < 32 ? 16 : 32); ++j) part[(int64_t)(c + j) * a.n_pad] = v[j];
      }
      __threadfence();
      named_bar_sync(1, 128);
      int* ticket = a.tickets + n_tile * a.m_tiles + m_tile;
      if (threadIdx.x == kEpiWarp0 * 32) last_s = atomicAdd(ticket, 1) == a.splits - 1;
      named_bar_sync(1, 128);
      if (last_s) {
        __threadfence();
        const float* base = a.partial + (int64_t)m0 * a.n_pad + n;
        const int64_t sstride = (int64_t)a.m_pad * a.n_pad;
#pragma unroll 1
        for (int j = 0; j < MT; ++j) {
          const int m = m0 + j;
          float acc = 0.f;
          for (int s = 0; s < a.splits; ++s) acc += __ldcg(base + s * sstride + (int64_t)j * a.n_pad);
          if (n < a.N && m < a.M) a.y[(int64_t)m * a.ldy + n] = __float2bfloat16_rn(acc);
        }
        if (threadIdx.x == kEpiWarp0 * 32) *ticket = 0;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_d), "r"(C::kTmemCols) : "memory");
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

int encode_2d(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  auto enc = encoder();
  if (!enc) return set_error(kNoEncoder, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(kEncode, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
  return kOk;
}

int pick_mt(int M) {
  if (M <= 16) return 16;
  if (M <= 32) return 32;
  if (M <= 64) return 64;
  if (M <= 128) return 128;
  return 256;
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!cached[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

struct Plan {
  int mt, n_tiles, m_tiles, splits, kb_total, kb_per_split, n_pad, m_pad;
  size_t ws_bytes;
};

// Split count from a two-term cost model: a split-K plan with s parts runs
// tiles*s CTAs in ceil(tiles*s / slots) waves; its time is the larger of
// (all bytes it moves) / HBM bandwidth and (waves x bytes one CTA streams) /
// per-SM streaming bandwidth. fp32 partials (s > 1) count at L2 bandwidth.
Plan make_plan(int M, int N, int K, int splits_req) {
  Plan p;
  p.mt = pick_mt(M);
  p.n_tiles = (N + kBN - 1) / kBN;
  p.m_tiles = (M + p.mt - 1) / p.mt;
  p.kb_total = (K + kBK - 1) / kBK;
  const int per_sm = p.mt <= 64 ? 2 : 1;
  const int slots = sm_count() * per_sm;
  const int tiles = p.n_tiles * p.m_tiles;
  int best = 1;
  if (splits_req > 0) {
    best = splits_req;
  } else {
    const double hbm = 6.5e12, l2 = 20e12, per_sm_bw = 60e9;
    double best_t = 1e30;
    const int max_s = p.kb_total / 4 > 1 ? p.kb_total / 4 : 1;
    for (int s = 1; s <= 32 && s <= max_s; ++s) {
      const int kb = (p.kb_total + s - 1) / s;
      const int se = (p.kb_total + kb - 1) / kb;
      const double unit = (double)(kBN + p.mt) * kb * kBK * 2;
      const double part = se > 1 ? 2.0 * p.mt * kBN * 4 : 0.0;
      const int units = tiles * se;
      const int waves = (units + slots - 1) / slots;
      const double t_mem = (double)units * unit / hbm + (double)units * part / l2;
      const double t_sm = (double)waves * (unit + part) / per_sm_bw;
      const double t = t_mem > t_sm ? t_mem : t_sm;
      if (t < best_t * 0.97) {
        best_t = t;
        best = se;
      }
    }
  }
  if (best > p.kb_total) best = p.kb_total;
  p.kb_per_split = (p.kb_total + best - 1) / best;
  p.splits = (p.kb_total + p.kb_per_split - 1) / p.kb_per_split;
  p.n_pad = p.n_tiles * kBN;
  p.m_pad = p.m_tiles * p.mt;
  p.ws_bytes = 0;
  if (p.splits > 1) {
    const size_t tick = ((size_t)tiles * sizeof(int) + 255) & ~size_t(255);
    p.ws_bytes = tick + (size_t)p.splits * p.m_pad * p.n_pad * sizeof(float);
  }
  return p;
}

template <int MT>
int launch(const CUtensorMap& wmap, const CUtensorMap& xmap, GemmArgs& a, cudaStream_t stream) {
  using C = Cfg<MT>;
  static unsigned long long done = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !((done >> dev) & 1ull)) {
    cudaError_t e = cudaFuncSetAttribute(gemm_kernel<MT>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    if (e != cudaSuccess) return cuda_status(e, "gemm smem attribute");
    if (dev < 64) done |= 1ull << dev;
  }
  a.idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(MT >> 3) << 17) | ((uint32_t)(kBN >> 4) << 24);
  const unsigned grid = (unsigned)(a.n_tiles * a.m_tiles * a.splits);
  gemm_kernel<MT><<<grid, kThreads, C::kSmem, stream>>>(wmap, xmap, a);
  return cuda_status(cudaGetLastError(), "kvb_gemm_bf16 launch");
}

}  // namespace
}  // namespace kvb

using namespace kvb;

extern "C" int kvb_gemm_workspace_size(int M, int N, int K, int splits, size_t* bytes) {
  if (!bytes || M < 0 || N <= 0 || K <= 0 || splits < 0) return set_error(kInvalid, "kvb_gemm_workspace_size: bad sizes");
  *bytes = M == 0 ? 0 : make_plan(M, N, K, splits).ws_bytes;
  return kOk;
}

extern "C" int kvb_gemm_bf16(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy, int M,
                             int N, int K, int splits, void* workspace, size_t workspace_bytes, void* stream) {
  if (M < 0 || N <= 0 || K <= 0 || splits < 0 || ldx < K || ldw < K || ldy < N)
    return set_error(kInvalid, "kvb_gemm_bf16: bad sizes or leading dimensions");
  if (M == 0) return kOk;
  if (!x || !w || !y) return set_error(kInvalid, "kvb_gemm_bf16: NULL pointer");
  if (((uintptr_t)x & 15) || ((uintptr_t)w & 15) || ldx % 8 || ldw % 8 || K % 8)
    return set_error(kInvalid, "kvb_gemm_bf16: x/w rows must be 16-byte aligned (K, ldx, ldw multiples of 8)");
  Plan p = make_plan(M, N, K, splits);
  if (p.ws_bytes > 0 && (!workspace || workspace_bytes < p.ws_bytes || ((uintptr_t)workspace & 255)))
    return set_error(kWorkspace, "kvb_gemm_bf16: workspace of %zu bytes (256-byte aligned, tickets zeroed) needed, %zu given",
                     p.ws_bytes, workspace_bytes);
  CUtensorMap wmap, xmap;
  int rc = encode_2d(&wmap, w, N, K, ldw, kBN);
  if (rc) return rc;
  rc = encode_2d(&xmap, x, M, K, ldx, p.mt);
  if (rc) return rc;
  GemmArgs a;
  a.y = (bf16*)y;
  a.ldy = ldy;
  a.M = M;
  a.N = N;
  a.n_tiles = p.n_tiles;
  a.m_tiles = p.m_tiles;
  a.splits = p.splits;
  a.kb_total = p.kb_total;
  a.kb_per_split = p.kb_per_split;
  a.n_pad = p.n_pad;
  a.m_pad = p.m_pad;
  const size_t tick = ((size_t)p.n_tiles * p.m_tiles * sizeof(int) + 255) & ~size_t(255);
  a.tickets = p.splits > 1 ? (int*)workspace : nullptr;
  a.partial = p.splits > 1 ? (float*)((uint8_t*)workspace + tick) : nullptr;
  cudaStream_t st = (cudaStream_t)stream;
  switch (p.mt) {
    case 16: return launch<16>(wmap, xmap, a, st);
    case 32: return launch<32>(wmap, xmap, a, st);
    case 64: return launch<64>(wmap, xmap, a, st);
    case 128: return launch<128>(wmap, xmap, a, st);
    default: return launch<256>(wmap, xmap, a, st);
  }
}
