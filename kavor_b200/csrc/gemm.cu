// bf16 GEMM on the 5th-generation tensor cores: Y[M, N] = X[M, K] * W[N, K]^T
// (F.linear of linear.py:50,73,157 and embed_head.py:61), fp32 accumulation in
// TMEM, bf16 output; and the gate-up projection fused with SiluAndMul.
//
// Orientation ("swap AB"): the UMMA A operand is a 128-row slab of the weight
// W (128 output features), the B operand is a tile of MT token rows of X, so
// the accumulator D[feature, token] lives in 128 TMEM lanes x MT columns. At
// decode batch sizes (M <= 256) the whole batch is one token tile and every
// weight byte is read from HBM exactly once.
//
// A CTA is warp-specialised:
//   warp 0      TMA producer: W box {64 K, 128 rows} (+ the up-half box when
//               gated) + X box {64 K, MT rows}, 128-byte swizzle, into a
//               `stages`-deep mbarrier ring;
//   warp 1      allocates TMEM; one thread issues
//               tcgen05.mma.cta_group::1.kind::f16 (M=128, N=MT, K=16) x4 per
//               stage (x8 gated), tcgen05.commit's each stage back to the
//               producer and each finished accumulator to the epilogue;
//   warps 2..5  epilogue, one TMEM lane quarter each (tcgen05.ld 32x32b).
//
// Two schedules, chosen with the tile MT by a cost model:
//   persistent  (no K split): CTAs walk a static list of (weight slab, token
//               tile) units; two TMEM accumulators, so the MMAs of the next
//               unit overlap this unit's epilogue, which goes through a
//               per-warp shared-memory transpose and leaves as 64-byte token
//               rows;
//   cluster     (K split over C = 2..16 CTAs of one thread-block cluster, one
//               unit per CTA): when its MMAs are done every CTA pushes its fp32
//               accumulator through distributed shared memory into the CTAs
//               that own each slice of the tile's sixteen 8-feature groups
//               (16 / C groups each when C divides 16; the stage ring, idle by
//               then, is the landing buffer), and each owner sums the C parts
//               in cluster-rank order — deterministic — and writes bf16. No
//               global scratch memory and no atomics.
// Optionally (kvb_gemm_set_l2_prefetch) the producer also asks L2 for the
// weight K-steps a fixed distance ahead of its TMA loads, so the loads that
// fill the ring wait on L2 rather than HBM latency.
// No cluster multicast is used anywhere (multi-GPU safe).
#include <cudaTypedefs.h>

#include <atomic>

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
constexpr int kMaxCluster = 16;

struct GemmArgs {
  bf16* y;
  int64_t ldy;
  int M, N;
  int n_tiles, m_tiles, splits, kb_total, kb_per_split;
  int units;
  int up_row0;      // gated: first weight row of the up half (= output width)
  uint32_t idesc;
  int vec_out;      // y rows are 16-byte aligned
  int pf;           // weight K-steps to prefetch into L2 ahead of the TMA loads (0: none)
  int gmax;         // cluster split: most 8-feature groups any rank owns (ceil(16 / splits))
};

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}

// Ask for the box at (c0, c1) to be brought into L2 (no shared memory, no
// barrier): the weight stream reaches the later TMA loads from L2 instead of HBM.
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap* map, int c0, int c1) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1)
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

// ------------------------------------------------------------ cluster helpers
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Every thread of every CTA of the cluster; release/acquire orders the
// distributed-shared-memory stores around it.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t map_to_rank(uint32_t local_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster_v4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

// 32 (or 16) consecutive TMEM columns of this warp's 32 lanes -> registers.
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

constexpr int pow2_at_least(int v) {
  int p = 32;
  while (p < v) p <<= 1;
  return p;
}

// G (gated): every unit multiplies the token tile with TWO weight slabs — the
// gate rows [n0, n0+128) and the up rows [I + n0, I + n0 + 128) of the
// [gate | up] weight (linear.py:76-93 layout) — into two accumulators, and the
// epilogue writes bf16(silu(gate) * up) (activation.py:8-11).
// CL (cluster split-K): one unit per CTA, one accumulator.
template <int MT, bool G, bool CL>
struct Cfg {
  static constexpr int kA = G ? 2 : 1;                      // weight slabs per unit
  static constexpr int kBBytes = MT * kBK * 2;
  static constexpr int kStageBytes = kA * kABytes + kBBytes;
  static constexpr int kPerSm = (!G && MT <= 64) ? 2 : 1;   // CTAs resident per SM
  static constexpr int kBudget = kPerSm == 2 ? 96 * 1024 : 192 * 1024;
  static constexpr int kStagesRaw = kBudget / kStageBytes;
  static constexpr int kStages = kStagesRaw > 8 ? 8 : (kStagesRaw < 2 ? 2 : kStagesRaw);
  static constexpr int kChunk = MT < 32 ? 16 : 32;          // tokens per TMEM load
  static constexpr int kOutBytes = CL ? 0 : 4 * 32 * kChunk * 2;  // per-warp transpose tiles
  static constexpr int kAccCols = kA * MT;                  // one accumulator (gate [+ up])
  static constexpr int kTmemCols = pow2_at_least(CL ? kAccCols : 2 * kAccCols);
  static constexpr int kPitch = MT + 4;                     // fp32 row pitch of the cluster landing buffer
  static constexpr int kRedBytes = kA * kBN * kPitch * 4;   // [slab][rank][feature/C][kPitch], any C
  static constexpr int kSmem = kStages * kStageBytes + kOutBytes + 1024;
  static_assert(!CL || kRedBytes <= kStages * kStageBytes, "landing buffer must fit the stage ring");
};

__device__ __forceinline__ float silu_mul_rounded(float g, float u) {
  // the reference rounds the projection to bf16 before SiluAndMul
  g = bf16_round(g);
  u = bf16_round(u);
  return g / (1.f + __expf(-g)) * u;
}

__device__ __forceinline__ void unit_coords(const GemmArgs& a, int u, int& n_tile, int& m_tile, int& split, int& kb0,
                                            int& nkb) {
  split = u % a.splits;  // = %cluster_ctarank in the cluster schedule (cluster dims {splits, 1, 1})
  const int t = u / a.splits;
  m_tile = t % a.m_tiles;
  n_tile = t / a.m_tiles;
  kb0 = split * a.kb_per_split;
  nkb = max(0, min(kb0 + a.kb_per_split, a.kb_total) - kb0);
}

template <int MT, bool G, bool CL>
__global__ void __launch_bounds__(kThreads, Cfg<MT, G, CL>::kPerSm)
    gemm_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                const __grid_constant__ GemmArgs a) {
  using C = Cfg<MT, G, CL>;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[S];
  __shared__ __align__(8) uint64_t empty_bar[S];
  __shared__ __align__(8) uint64_t acc_full[2];
  __shared__ __align__(8) uint64_t acc_empty[2];
  __shared__ uint32_t tmem_base_s;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&acc_full[b]), 1);
      mbar_init(smem_u32(&acc_empty[b]), 4);
    }
    fence_barrier_init();
  }
  // Launched programmatically (kvb_set_pdl), this kernel may start while the
  // kernel before it still runs: the weights are not that kernel's output, so
  // the producer (thread 0) requests the weight tiles of its first unit's first
  // K-steps into the stage ring now, and only the token tiles wait for the
  // grid dependency. Without programmatic launch nothing is issued early.
  int pre = 0;  // K-steps whose weight tiles are already requested (thread 0)
  if (threadIdx.x == 0 && c_pdl_trigger && (int)blockIdx.x < a.units) {
    prefetch_tensormap(&wmap);
    int n_tile, m_tile, split, kb0, nkb;
    unit_coords(a, blockIdx.x, n_tile, m_tile, split, kb0, nkb);
    pre = nkb < S ? nkb : S;
    for (int i = 0; i < pre; ++i) {
      const uint32_t sa = smem_u32(smem + i * C::kStageBytes);
      const uint32_t fb = smem_u32(&full_bar[i]);
      mbar_arrive_expect_tx(fb, C::kStageBytes);
      tma_load_2d(sa, &wmap, (kb0 + i) * kBK, n_tile * kBN, fb);
      if constexpr (G) tma_load_2d(sa + kABytes, &wmap, (kb0 + i) * kBK, a.up_row0 + n_tile * kBN, fb);
    }
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
  kernel_entry();  // the token tiles and every output row come after the grid dependency
  const uint32_t tmem = tmem_base_s;
  bool dead = false;  // a bounded wait gave up: skip the work, keep every barrier balanced

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      prefetch_tensormap(&wmap);
      prefetch_tensormap(&xmap);
      int it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < a.units && ok; u += gridDim.x) {
        int n_tile, m_tile, split, kb0, nkb;
        unit_coords(a, u, n_tile, m_tile, split, kb0, nkb);
        // weight K-steps [first, pf) go to L2 now, step i + pf after step i's
        // load; the first S steps of the CTA's first unit are loaded at once
        const int first = u == (int)blockIdx.x ? S : 0;
        for (int j = first; j < a.pf && j < nkb; ++j) {
          tma_prefetch_l2_2d(&wmap, (kb0 + j) * kBK, n_tile * kBN);
          if constexpr (G) tma_prefetch_l2_2d(&wmap, (kb0 + j) * kBK, a.up_row0 + n_tile * kBN);
        }
        for (int i = 0; i < nkb; ++i, ++it) {
          const int s = it % S;
          if (it >= S && !mbar_wait(smem_u32(&empty_bar[s]), ((it / S) - 1) & 1, &g_err_gemm)) {
            ok = false;
            break;
          }
          const uint32_t sa = smem_u32(smem + s * C::kStageBytes);
          const uint32_t fb = smem_u32(&full_bar[s]);
          if (it >= pre) {  // (the first `pre` steps' weights were requested before the grid dependency)
            mbar_arrive_expect_tx(fb, C::kStageBytes);
            tma_load_2d(sa, &wmap, (kb0 + i) * kBK, n_tile * kBN, fb);
            if constexpr (G) tma_load_2d(sa + kABytes, &wmap, (kb0 + i) * kBK, a.up_row0 + n_tile * kBN, fb);
          }
          tma_load_2d(sa + C::kA * kABytes, &xmap, (kb0 + i) * kBK, m_tile * MT, fb);
          const int j = i + a.pf;
          if (a.pf > 0 && j < nkb && j >= first) {
            tma_prefetch_l2_2d(&wmap, (kb0 + j) * kBK, n_tile * kBN);
            if constexpr (G) tma_prefetch_l2_2d(&wmap, (kb0 + j) * kBK, a.up_row0 + n_tile * kBN);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int it = 0, local = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < a.units && ok; u += gridDim.x, ++local) {
        int n_tile, m_tile, split, kb0, nkb;
        unit_coords(a, u, n_tile, m_tile, split, kb0, nkb);
        const int buf = local & 1;
        if (local >= 2 && !mbar_wait(smem_u32(&acc_empty[buf]), ((local >> 1) - 1) & 1, &g_err_gemm)) break;
        tc_fence_after();
        const uint32_t d = tmem + buf * C::kAccCols;
        for (int i = 0; i < nkb; ++i, ++it) {
          const int s = it % S;
          if (!mbar_wait(smem_u32(&full_bar[s]), (it / S) & 1, &g_err_gemm)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * C::kStageBytes);
          const uint64_t da = smem_desc_sw128(sa), db = smem_desc_sw128(sa + C::kA * kABytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)  // +32 bytes along K inside the swizzle atom = +2 in the address field
            umma_bf16(d, da + 2 * k, db + 2 * k, a.idesc, (i > 0 || k > 0) ? 1u : 0u);
          if constexpr (G) {
            const uint64_t du = smem_desc_sw128(sa + kABytes);
#pragma unroll
            for (int k = 0; k < kBK / 16; ++k)
              umma_bf16(d + MT, du + 2 * k, db + 2 * k, a.idesc, (i > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(smem_u32(&empty_bar[s]));
        }
        umma_commit(smem_u32(&acc_full[buf]));
      }
      // no MMA may still run when TMEM is freed (or, clustered, when the ring
      // becomes a landing buffer): wait for the last accumulator
      if (local > 0) mbar_wait(smem_u32(&acc_full[(local - 1) & 1]), ((local - 1) >> 1) & 1, &g_err_gemm);
    }
  } else if constexpr (!CL) {
    // ---------------------------------------------------------------- epilogue (persistent)
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    constexpr int CH = C::kChunk;
    bf16* tile_out = reinterpret_cast<bf16*>(smem + S * C::kStageBytes) + (warp - kEpiWarp0) * 32 * CH;
    int local = 0;
    for (int u = blockIdx.x; u < a.units; u += gridDim.x, ++local) {
      int n_tile, m_tile, split, kb0, nkb;
      unit_coords(a, u, n_tile, m_tile, split, kb0, nkb);
      const int buf = local & 1;
      const int n0 = n_tile * kBN, m0 = m_tile * MT;
      if (!dead && !mbar_wait(smem_u32(&acc_full[buf]), (local >> 1) & 1, &g_err_gemm)) dead = true;
      if (dead) continue;
      tc_fence_after();
      const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16) + buf * C::kAccCols;
#pragma unroll 1
      for (int c = 0; c < MT; c += CH) {
        float v[32];
        if constexpr (CH == 16) tmem_ld16(trow + c, v); else tmem_ld32(trow + c, v);
        if constexpr (G) {
          float w[32];
          if constexpr (CH == 16) tmem_ld16(trow + MT + c, w); else tmem_ld32(trow + MT + c, w);
#pragma unroll
          for (int j = 0; j < CH; ++j) v[j] = silu_mul_rounded(v[j], w[j]);
        }
        // transpose through shared memory: tile_out[token][feature], 64-byte rows
#pragma unroll
        for (int j = 0; j < CH; ++j) tile_out[j * 32 + lane] = __float2bfloat16_rn(v[j]);
        __syncwarp();
        const int m = m0 + c + lane;
        const int nb = n0 + q * 32;
        if (lane < CH && m < a.M) {
          bf16* yr = a.y + (int64_t)m * a.ldy + nb;
          const bf16* src = tile_out + lane * 32;
          if (a.vec_out && nb + 32 <= a.N) {
#pragma unroll
            for (int e = 0; e < 4; ++e) reinterpret_cast<uint4*>(yr)[e] = reinterpret_cast<const uint4*>(src)[e];
          } else {
            for (int e = 0; e < 32 && nb + e < a.N; ++e) yr[e] = src[e];
          }
        }
        __syncwarp();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&acc_empty[buf]));
    }
  } else {
    // ---------------------------------------------------------------- epilogue (cluster), part 1
    if (!mbar_wait(smem_u32(&acc_full[0]), 0, &g_err_gemm)) dead = true;
    tc_fence_after();
  }

  if constexpr (CL) {
    // part 2: every CTA's MMAs are complete after this barrier, so every stage
    // ring is free; push the fp32 accumulator slices to their owners
    __syncwarp();
    cluster_sync_all();
    // The tile's 16 groups of 8 features are dealt to the C ranks in order,
    // rank o owning groups [16 o / C, 16 (o + 1) / C) (128 / C features each
    // when C divides 16). The landing buffer holds, per slab and source rank,
    // gmax groups of 8 rows of kPitch floats.
    const int Cn = a.splits;
    const int rows_per_src = a.gmax * 8;
    const uint32_t rank = cluster_rank();
    const bool fits = C::kA * Cn * rows_per_src * C::kPitch * 4 <= S * C::kStageBytes;  // the host plan ensures it
    if (!fits && threadIdx.x == 0) atomicOr(&g_err_gemm, (unsigned)kErrConfig);
    int n_tile, m_tile, split, kb0, nkb;
    unit_coords(a, blockIdx.x, n_tile, m_tile, split, kb0, nkb);
    const uint32_t red = smem_u32(smem);
    if (warp >= kEpiWarp0 && !dead && fits) {
      constexpr int CH = C::kChunk;
      const int q = warp & 3;
      const int f = q * 32 + lane;
      const int grp = f >> 3;
      const int owner = ((grp + 1) * Cn + 15) / 16 - 1;
      const int fl = (grp - owner * 16 / Cn) * 8 + (f & 7);  // row inside the owner's part
      const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
      for (int h = 0; h < C::kA; ++h) {
        const uint32_t dst =
            map_to_rank(red + (uint32_t)((((h * Cn + (int)rank) * rows_per_src + fl) * C::kPitch) * 4), (uint32_t)owner);
#pragma unroll 1
        for (int c = 0; c < MT; c += CH) {
          float v[32];
          if (nkb > 0) {
            if constexpr (CH == 16) tmem_ld16(trow + h * MT + c, v); else tmem_ld32(trow + h * MT + c, v);
          } else {
#pragma unroll
            for (int j = 0; j < CH; ++j) v[j] = 0.f;
          }
#pragma unroll
          for (int j = 0; j < CH; j += 4) st_cluster_v4(dst + (uint32_t)(c + j) * 4, v[j], v[j + 1], v[j + 2], v[j + 3]);
        }
      }
    }
    tc_fence_before();
    __syncwarp();
    cluster_sync_all();
    // part 3: this CTA owns feature groups [g0, g0 + ng) of the tile
    if (warp >= kEpiWarp0 && !dead && fits) {
      const float* rf = reinterpret_cast<const float*>(smem);
      const int e = threadIdx.x - kEpiWarp0 * 32;
      const int g0 = (int)rank * 16 / Cn, ng = ((int)rank + 1) * 16 / Cn - g0;
      const int groups = ng * MT;
      const int n0 = n_tile * kBN + g0 * 8, m0 = m_tile * MT;
#pragma unroll 1
      for (int g = e; g < groups; g += 128) {
        const int ml = g % MT, fg = g / MT;
        const int m = m0 + ml;
        if (m >= a.M) continue;
        float acc[8], acu[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = acu[j] = 0.f;
#pragma unroll 1
        for (int s = 0; s < Cn; ++s) {
          const float* p = rf + ((s * rows_per_src + fg * 8) * C::kPitch + ml);
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[j] += p[j * C::kPitch];
          if constexpr (G) {
            const float* pu = p + Cn * rows_per_src * C::kPitch;
#pragma unroll
            for (int j = 0; j < 8; ++j) acu[j] += pu[j * C::kPitch];
          }
        }
        if constexpr (G) {
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[j] = silu_mul_rounded(acc[j], acu[j]);
        }
        const int n = n0 + fg * 8;
        bf16* yr = a.y + (int64_t)m * a.ldy + n;
        if (a.vec_out && n + 8 <= a.N) {
          uint4 pk;
          __nv_bfloat162* h2 = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
          for (int j = 0; j < 4; ++j) h2[j] = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
          *reinterpret_cast<uint4*>(yr) = pk;
        } else {
          for (int j = 0; j < 8 && n + j < a.N; ++j) yr[j] = __float2bfloat16_rn(acc[j]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::kTmemCols) : "memory");
  }
}

int encode_2d(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  auto enc = tensor_map_encoder();
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

// K-steps of weight the producer asks L2 for ahead of its TMA loads
// (kvb_gemm_set_l2_prefetch; 0 = off).
std::atomic<int> g_l2_prefetch{0};

struct Plan {
  int mt, n_tiles, m_tiles, splits, kb_total, kb_per_split, units, grid;
};

struct TileShape {
  int mt, stages, per_sm;
};

constexpr TileShape kShapes[] = {{16, Cfg<16, false, false>::kStages, Cfg<16, false, false>::kPerSm},
                                 {32, Cfg<32, false, false>::kStages, Cfg<32, false, false>::kPerSm},
                                 {64, Cfg<64, false, false>::kStages, Cfg<64, false, false>::kPerSm},
                                 {128, Cfg<128, false, false>::kStages, Cfg<128, false, false>::kPerSm},
                                 {256, Cfg<256, false, false>::kStages, Cfg<256, false, false>::kPerSm}};
constexpr TileShape kGatedShapes[] = {{16, Cfg<16, true, false>::kStages, Cfg<16, true, false>::kPerSm},
                                      {32, Cfg<32, true, false>::kStages, Cfg<32, true, false>::kPerSm},
                                      {64, Cfg<64, true, false>::kStages, Cfg<64, true, false>::kPerSm},
                                      {128, Cfg<128, true, false>::kStages, Cfg<128, true, false>::kPerSm}};

// The cluster split's landing buffer (the stage ring) holds, per weight slab
// and source rank, ceil(16 / C) groups of 8 feature rows of (mt + 4) floats.
bool landing_fits(int mt, bool gated, int stages, int splits) {
  if (splits <= 1) return true;
  const int slabs = gated ? 2 : 1;
  const int64_t rows = (int64_t)slabs * splits * ((16 + splits - 1) / splits) * 8;
  const int64_t ring = (int64_t)stages * (slabs * kABytes + mt * kBK * 2);
  return rows * (mt + 4) * 4 <= ring;
}

Plan finish_plan(int M, int N, int K, int mt, int per_sm, int splits) {
  Plan p;
  p.mt = mt;
  p.n_tiles = (N + kBN - 1) / kBN;
  p.m_tiles = (M + mt - 1) / mt;
  p.kb_total = (K + kBK - 1) / kBK;
  if (splits > p.kb_total) splits = p.kb_total;
  if (splits > kMaxCluster) splits = kMaxCluster;
  if (splits < 1) splits = 1;
  p.splits = splits;
  p.kb_per_split = (p.kb_total + splits - 1) / splits;
  p.units = p.n_tiles * p.m_tiles * p.splits;
  const int slots = device_sm_count() * per_sm;
  p.grid = (p.splits > 1 || p.units < slots) ? p.units : slots;
  return p;
}

// Cost model (microseconds). Per K-block a CTA is bound by the tensor pipe
// (4 MMAs of 128 x MT x 16 per weight slab, 128 cycles each at MT = 256) or by
// what it can pull through TMA (~200 GB/s per SM); a CTA also pays a pipeline
// fill. Persistent: ceil(units / grid) units back to back, epilogues hidden
// except the last. Cluster: waves of clusters, each paying the DSMEM exchange
// (~60 GB/s per SM) and the reduction. The whole GEMM is also bound by HBM:
// the weight once per token tile (no reuse across tiles is assumed), the
// tokens and the output.
double plan_cost(const Plan& p, int M, int N, int K, int per_sm, int slabs) {
  const double clk = 1.9e3;  // cycles per us
  const int nsm = device_sm_count();
  const double t_mma = 4.0 * slabs * 128.0 * (p.mt < 32 ? 32 : p.mt) / 256.0 / clk;
  const double kb_bytes = slabs * (double)kABytes + (double)p.mt * kBK * 2;
  const double t_tma = kb_bytes / (per_sm == 2 ? 120e3 : 200e3);
  const double t_kb = t_mma > t_tma ? t_mma : t_tma;
  const double fill = 1.2;
  double t_cta;
  if (p.splits == 1) {
    const int upc = (p.units + p.grid - 1) / p.grid;
    t_cta = fill + upc * p.kb_per_split * t_kb + p.mt * kBN * 2.0 / 150e3;
  } else {
    const int per_wave = (nsm * per_sm / p.splits) * p.splits;
    const int waves = (p.units + per_wave - 1) / per_wave;
    const double xchg = slabs * 128.0 * p.mt * 4.0 * (p.splits - 1) / p.splits / 60e3 + 0.5;
    t_cta = waves * (fill + p.kb_per_split * t_kb + xchg);
  }
  const double hbm = ((double)slabs * N * K * p.m_tiles + (double)M * K + (double)M * N) * 2.0 / 6.5e6;
  return t_cta > hbm ? t_cta : hbm;
}

// N is the OUTPUT width (for the gated form: the intermediate size I).
// splits_req > 0 forces the K split (cluster size 1..16; the automatic choice
// considers powers of two).
Plan make_plan(int M, int N, int K, int splits_req, bool gated = false) {
  Plan best{};
  double best_t = 1e30;
  const int slabs = gated ? 2 : 1;
  const TileShape* shapes = gated ? kGatedShapes : kShapes;
  const int nshapes = gated ? 4 : 5;
  static const int kSplits[] = {1, 2, 4, 8, 16};
  const int forced[] = {splits_req};
  const int* cand = splits_req > 0 ? forced : kSplits;
  const int ncand = splits_req > 0 ? 1 : 5;
  for (int si = 0; si < nshapes; ++si) {
    const TileShape& sh = shapes[si];
    if (sh.mt > 16 && sh.mt >= 2 * M) continue;  // a token tile far above the batch wastes tensor work
    for (int ci = 0; ci < ncand; ++ci) {
      const int s = cand[ci];
      Plan p = finish_plan(M, N, K, sh.mt, sh.per_sm, s);
      if (p.splits != s) continue;
      if (p.splits > 1 && (int64_t)(p.splits - 1) * p.kb_per_split >= p.kb_total) continue;  // an empty part
      if (!landing_fits(sh.mt, gated, sh.stages, p.splits)) continue;
      const double t = plan_cost(p, M, N, K, sh.per_sm, slabs);
      if (t < best_t * 0.97) {
        best_t = t;
        best = p;
      }
    }
  }
  if (best.mt == 0) {  // a forced split that no tile accepts: fall back to the heuristic
    return make_plan(M, N, K, 0, gated);
  }
  return best;
}

template <int MT, bool G, bool CL>
int launch(const CUtensorMap& wmap, const CUtensorMap& xmap, GemmArgs& a, int grid, cudaStream_t stream) {
  using C = Cfg<MT, G, CL>;
  static unsigned long long done = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !((done >> dev) & 1ull)) {
    cudaError_t e = cudaFuncSetAttribute(gemm_kernel<MT, G, CL>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    if (e == cudaSuccess && CL)
      e = cudaFuncSetAttribute(gemm_kernel<MT, G, CL>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return cuda_status(e, "gemm kernel attributes");
    if (dev < 64) done |= 1ull << dev;
  }
  a.idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(MT >> 3) << 17) | ((uint32_t)(kBN >> 4) << 24);
  if constexpr (!CL) {
    return cuda_status(launch_kernel(gemm_kernel<MT, G, CL>, dim3(grid), dim3(kThreads), C::kSmem, stream, wmap, xmap,
                                     a),
                       "kvb_gemm launch");
  } else {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = C::kSmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = a.splits;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    return cuda_status(cudaLaunchKernelEx(&cfg, gemm_kernel<MT, G, CL>, wmap, xmap, a), "kvb_gemm cluster launch");
  }
}

template <int MT, bool G>
int launch_mt(const CUtensorMap& wmap, const CUtensorMap& xmap, GemmArgs& a, int grid, cudaStream_t stream) {
  return a.splits > 1 ? launch<MT, G, true>(wmap, xmap, a, grid, stream) : launch<MT, G, false>(wmap, xmap, a, grid, stream);
}

// y[M, n_out] = x w^T (gated: bf16(silu(x w_gate^T) * (x w_up^T)), w = [gate | up]
// with n_out rows each).
int run_gemm(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy, int M, int n_out, int K,
             int splits, void* stream, bool gated, const char* name) {
  if (M < 0 || n_out <= 0 || K <= 0 || splits < 0 || ldx < K || ldw < K || ldy < n_out)
    return set_error(kInvalid, "%s: bad sizes or leading dimensions", name);
  if (M == 0) return kOk;
  if (!x || !w || !y) return set_error(kInvalid, "%s: NULL pointer", name);
  if (((uintptr_t)x & 15) || ((uintptr_t)w & 15) || ldx % 8 || ldw % 8 || K % 8)
    return set_error(kInvalid, "%s: x/w rows must be 16-byte aligned (K, ldx, ldw multiples of 8)", name);
  Plan p = make_plan(M, n_out, K, splits, gated);
  CUtensorMap wmap, xmap;
  int rc = encode_2d(&wmap, w, (int64_t)n_out * (gated ? 2 : 1), K, ldw, kBN);
  if (rc) return rc;
  rc = encode_2d(&xmap, x, M, K, ldx, p.mt);
  if (rc) return rc;
  GemmArgs a;
  a.y = (bf16*)y;
  a.ldy = ldy;
  a.M = M;
  a.N = n_out;
  a.n_tiles = p.n_tiles;
  a.m_tiles = p.m_tiles;
  a.splits = p.splits;
  a.kb_total = p.kb_total;
  a.kb_per_split = p.kb_per_split;
  a.units = p.units;
  a.up_row0 = n_out;
  a.vec_out = ((uintptr_t)y & 15) == 0 && ldy % 8 == 0;
  a.pf = g_l2_prefetch.load(std::memory_order_relaxed);
  a.gmax = (16 + p.splits - 1) / p.splits;
  cudaStream_t st = (cudaStream_t)stream;
  if (gated) {
    switch (p.mt) {
      case 16: return launch_mt<16, true>(wmap, xmap, a, p.grid, st);
      case 32: return launch_mt<32, true>(wmap, xmap, a, p.grid, st);
      case 64: return launch_mt<64, true>(wmap, xmap, a, p.grid, st);
      default: return launch_mt<128, true>(wmap, xmap, a, p.grid, st);
    }
  }
  switch (p.mt) {
    case 16: return launch_mt<16, false>(wmap, xmap, a, p.grid, st);
    case 32: return launch_mt<32, false>(wmap, xmap, a, p.grid, st);
    case 64: return launch_mt<64, false>(wmap, xmap, a, p.grid, st);
    case 128: return launch_mt<128, false>(wmap, xmap, a, p.grid, st);
    default: return launch_mt<256, false>(wmap, xmap, a, p.grid, st);
  }
}

}  // namespace
}  // namespace kvb

using namespace kvb;

extern "C" int kvb_gemm_workspace_size(int M, int N, int K, int splits, size_t* bytes) {
  if (!bytes || M < 0 || N <= 0 || K <= 0 || splits < 0) return set_error(kInvalid, "kvb_gemm_workspace_size: bad sizes");
  *bytes = 0;  // the K split reduces through distributed shared memory
  return kOk;
}

extern "C" int kvb_gemm_bf16(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy, int M,
                             int N, int K, int splits, void* workspace, size_t workspace_bytes, void* stream) {
  (void)workspace;
  (void)workspace_bytes;
  return run_gemm(x, ldx, w, ldw, y, ldy, M, N, K, splits, stream, false, "kvb_gemm_bf16");
}

extern "C" int kvb_gemm_silu_workspace_size(int M, int inter, int K, int splits, size_t* bytes) {
  if (!bytes || M < 0 || inter <= 0 || K <= 0 || splits < 0)
    return set_error(kInvalid, "kvb_gemm_silu_workspace_size: bad sizes");
  *bytes = 0;
  return kOk;
}

extern "C" int kvb_gemm_silu_bf16(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy, int M,
                                  int inter, int K, int splits, void* workspace, size_t workspace_bytes, void* stream) {
  (void)workspace;
  (void)workspace_bytes;
  return run_gemm(x, ldx, w, ldw, y, ldy, M, inter, K, splits, stream, true, "kvb_gemm_silu_bf16");
}

extern "C" int kvb_gemm_set_l2_prefetch(int ksteps) {
  if (ksteps < 0 || ksteps > 64) return set_error(kInvalid, "kvb_gemm_set_l2_prefetch: ksteps must be in [0, 64]");
  g_l2_prefetch.store(ksteps, std::memory_order_relaxed);
  return kOk;
}

extern "C" int kvb_gemm_plan(int M, int N, int K, int splits, int gated, int* plan) {
  if (!plan || M <= 0 || N <= 0 || K <= 0 || splits < 0) return set_error(kInvalid, "kvb_gemm_plan: bad sizes");
  const Plan p = make_plan(M, N, K, splits, gated != 0);
  plan[0] = p.mt;
  plan[1] = p.splits;
  plan[2] = p.units;
  plan[3] = p.grid;
  return kOk;
}
