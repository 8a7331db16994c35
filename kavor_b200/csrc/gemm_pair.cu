// bf16 GEMM on CTA pairs (tcgen05 cta_group::2): Y[M, N] = X[M, K] W[N, K]^T
// (F.linear of linear.py:50,73,157), fp32 accumulation in TMEM, bf16 output.
// The decode-batch form of the projection (M up to 256 tokens per tile):
//
// * two CTAs of a cluster form a pair; one tcgen05.mma.cta_group::2 of
//   M = 256 weight rows (128 in each CTA's shared memory) x N = MT tokens
//   (MT/2 token rows in each CTA) x K = 16, issued by one thread of the even
//   CTA, accumulates each CTA's 128 weight rows into its own TMEM. Per 64-wide
//   K step a CTA stages 16 KB of weight and MT/2 x 128 B of tokens: a
//   256-token tile moves 32 KB per SM per K step where a single-CTA tile of
//   128 weight rows moves 48 KB for the same MMA work;
// * both CTAs' TMA loads (.cta_group::2, no multicast) complete on the even
//   CTA's full barrier (it expects both CTAs' bytes); the MMA thread's
//   tcgen05.commit multicasts the stage release to both CTAs' empty barriers
//   and the final accumulator commit to both CTAs' accumulator barriers;
// * the K dimension is split over `splits` pairs of the same cluster (cluster
//   of 2 x splits CTAs): each CTA pushes its fp32 accumulator through
//   distributed shared memory into the CTAs of the same pair position that
//   own each slice of its sixteen 8-feature groups, and the owner sums the
//   parts in split order (deterministic) and writes bf16 rows of 8 features;
// * warp 0 issues TMA, warp 1 holds the pair's TMEM allocation and (even CTA)
//   issues the MMAs, warps 2..5 read TMEM (one lane quarter each).
// Every wait is bounded (kSpinCycles): a wait that gives up sets the error
// word and the CTA skips its remaining work, keeping every cluster barrier.
#include <cudaTypedefs.h>

#include <atomic>

#include "common.cuh"
#include "tcgen05.cuh"
#include "../../include/kavor_b200.h"

KVB_DEFINE_ERROR_WORD(gemm_pair)

namespace kvb {
namespace {

constexpr int kBK = 64;           // K elements per stage = one 128-byte swizzle row
constexpr int kSlab = 128;        // weight rows per CTA (half of the pair's UMMA M)
constexpr int kThreads = 192;     // 6 warps
constexpr int kEpiWarp0 = 2;
constexpr int kMaxSplits = 8;     // clusters of at most 16 CTAs

struct PairArgs {
  bf16* y;
  int64_t ldy;
  int M, N;
  int n_tiles;      // tiles of 2 x 128 weight rows
  int m_tiles;      // tiles of MT tokens
  int splits, kb_total, kb_per_split;
  int gmax;         // most 8-feature groups a split rank owns: ceil(16 / splits)
  uint32_t idesc;
  int vec_out;      // y rows are 16-byte aligned
  int up_row0;      // gated: first weight row of the up half (= the output width I)
};

template <int MT>
struct PairCfg {
  static constexpr int kHalf = MT / 2;                   // token rows each CTA of the pair loads
  static constexpr int kABytes = kSlab * kBK * 2;        // 16 KB
  static constexpr int kBBytes = kHalf * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStagesRaw = (192 * 1024) / kStageBytes;
  static constexpr int kStages = kStagesRaw > 8 ? 8 : kStagesRaw;
  static constexpr int kTmemCols = MT < 32 ? 32 : MT;    // one fp32 column per token (MT a power of two)
  static constexpr int kPitch = MT + 4;                  // fp32 row pitch of the landing buffer
  static constexpr int kUpPitch = MT + 8;                // bf16 row pitch of the gated form's up rows
  static constexpr int kSmem = kStages * kStageBytes + 1024;
  static_assert(MT == 64 || MT == 128 || MT == 256, "token tile");
  static_assert(kSmem <= 227 * 1024, "dynamic shared memory of one CTA");
  static_assert(kTmemCols <= 512, "TMEM columns of one SM");
};

// Landing buffer (the stage ring) of a K split: per source split, gmax groups
// of 8 feature rows of MT + 4 floats; the gated form adds the up owner's
// gmax x 8 bf16 rows of MT + 8.
template <int MT>
constexpr bool pair_landing_fits(int splits, bool gated) {
  const int64_t rows = (int64_t)((16 + splits - 1) / splits) * 8;
  return splits * rows * PairCfg<MT>::kPitch * 4 + (gated ? rows * PairCfg<MT>::kUpPitch * 2 : 0) <=
         (int64_t)PairCfg<MT>::kStages * PairCfg<MT>::kStageBytes;
}

// G (gated, splits = 1): a pair tile is 128 output features; the even CTA
// holds the gate rows [n0, n0 + 128) and the odd CTA the up rows
// [I + n0, I + n0 + 128) of the [gate | up] weight (linear.py:76-93 layout),
// so one pair MMA computes both halves; the odd CTA hands its up values
// (rounded to bf16, as the reference rounds the projection) to the even CTA
// through distributed shared memory, which writes bf16(silu(bf16(g)) * u)
// (activation.py:8-11).
template <int MT, bool G>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                     const __grid_constant__ PairArgs a) {
  kernel_entry();
  using C = PairCfg<MT>;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[S];
  __shared__ __align__(8) uint64_t empty_bar[S];
  __shared__ __align__(8) uint64_t acc_full;
  __shared__ uint32_t tmem_base_s;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const uint32_t rank = tc::cluster_rank();  // cluster = {2 x splits, 1, 1}: rank = blockIdx.x % (2 x splits)
  const int member = (int)(rank & 1u);       // 0: issues the pair's MMAs; 1: its peer
  const int split = (int)(rank >> 1);
  const int tile = (int)blockIdx.x / (2 * a.splits);
  const int m_tile = tile % a.m_tiles, n_tile = tile / a.m_tiles;
  const int kb0 = split * a.kb_per_split;
  const int nkb = max(0, min(kb0 + a.kb_per_split, a.kb_total) - kb0);
  // this CTA's weight rows = its rows of D
  const int n0 = G ? n_tile * kSlab + member * a.up_row0 : n_tile * 2 * kSlab + member * kSlab;
  const int mload = m_tile * MT + member * C::kHalf;    // token rows this CTA stages
  const uint16_t pair_mask = (uint16_t)(3u << (rank & ~1u));

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), 1);
    }
    mbar_init(smem_u32(&acc_full), 1);
    fence_barrier_init();
  }
  if (warp == 1) tc::tmem_alloc_pair(smem_u32(&tmem_base_s), C::kTmemCols);
  tc::fence_before();
  tc::cluster_sync_all();  // both CTAs' barriers exist before either signals the other's
  tc::fence_after();
  const uint32_t tmem = tmem_base_s;
  bool dead = false;  // a bounded wait gave up: skip the work, keep every barrier

  if (warp == 0) {
    // ---------------------------------------------------------------- producer (both CTAs)
    if (lane == 0) {
      prefetch_tensormap(&wmap);
      prefetch_tensormap(&xmap);
      const uint32_t leader = rank & ~1u;
      bool ok = true;
      for (int i = 0; i < nkb; ++i) {
        const int s = i % S;
        if (i >= S && !mbar_wait(smem_u32(&empty_bar[s]), ((i / S) - 1) & 1, &g_err_gemm_pair)) {
          ok = false;
          break;
        }
        const uint32_t sa = smem_u32(smem + s * C::kStageBytes);
        const uint32_t fb = smem_u32(&full_bar[s]);
        if (member == 0) mbar_arrive_expect_tx(fb, 2 * C::kStageBytes);  // this CTA's and the peer's bytes
        const uint32_t fb_leader = tc::map_to_rank(fb, leader);
        tc::tma_load_2d_pair(sa, &wmap, (kb0 + i) * kBK, n0, fb_leader);
        tc::tma_load_2d_pair(sa + C::kABytes, &xmap, (kb0 + i) * kBK, mload, fb_leader);
      }
      // the MMA thread's last stage releases land on this CTA's empty
      // barriers: wait for them before the ring is reused or the CTA exits
      for (int i = max(0, nkb - S); ok && i < nkb; ++i)
        ok = mbar_wait(smem_u32(&empty_bar[i % S]), (i / S) & 1, &g_err_gemm_pair);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer (even CTA)
    if (lane == 0 && member == 0) {
      bool ok = true;
      for (int i = 0; i < nkb; ++i) {
        const int s = i % S;
        if (!mbar_wait(smem_u32(&full_bar[s]), (i / S) & 1, &g_err_gemm_pair)) {
          ok = false;
          break;
        }
        tc::fence_after();
        const uint32_t sa = smem_u32(smem + s * C::kStageBytes);
        const uint64_t da = tc::smem_desc_sw128(sa), db = tc::smem_desc_sw128(sa + C::kABytes);
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k)  // +32 bytes along K inside the swizzle atom = +2 in the address field
          tc::umma_pair_bf16(tmem, da + 2 * k, db + 2 * k, a.idesc, (i > 0 || k > 0) ? 1u : 0u);
        tc::umma_commit_pair(smem_u32(&empty_bar[s]), pair_mask);
      }
      if (ok) {
        tc::umma_commit_pair(smem_u32(&acc_full), pair_mask);
        // no MMA may still read either ring when it becomes a landing buffer
        mbar_wait(smem_u32(&acc_full), 0, &g_err_gemm_pair);
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue, part 1 (both CTAs)
    if (!mbar_wait(smem_u32(&acc_full), 0, &g_err_gemm_pair)) dead = true;
    tc::fence_after();
  }

  if (G && a.splits == 1) {
    // the odd CTA's up rows, rounded to bf16, land in the even CTA's (free) ring
    __syncwarp();
    tc::cluster_sync_all();
    const int q = warp & 3;  // the TMEM lane quarter this warp may read
    const int f = q * 32 + lane;
    const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16);
    if (warp >= kEpiWarp0 && !dead && member == 1) {
      const uint32_t dst = tc::map_to_rank(smem_u32(smem) + (uint32_t)(f * C::kUpPitch * 2), rank & ~1u);
#pragma unroll 1
      for (int c = 0; c < MT; c += 32) {
        float v[32];
        tc::tmem_ld32(trow + c, v);
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          uint32_t w4[4];
#pragma unroll
          for (int h = 0; h < 4; ++h) w4[h] = pack_bf16(v[j + 2 * h], v[j + 2 * h + 1]);
          tc::st_cluster_v4(dst + (uint32_t)(c + j) * 2, __uint_as_float(w4[0]), __uint_as_float(w4[1]),
                            __uint_as_float(w4[2]), __uint_as_float(w4[3]));
        }
      }
    }
    tc::fence_before();
    __syncwarp();
    tc::cluster_sync_all();
    if (warp >= kEpiWarp0 && !dead && member == 0) {
      const bf16* up = reinterpret_cast<const bf16*>(smem) + f * C::kUpPitch;
      const int n = n0 + f, m0 = m_tile * MT;
      const bool in_range = n < a.up_row0;  // the last tile may reach past the I output features
#pragma unroll 1
      for (int c = 0; c < MT; c += 32) {
        float v[32];
        tc::tmem_ld32(trow + c, v);  // the whole warp, converged
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int m = m0 + c + j;
          if (in_range && m < a.M) {
            const float g = bf16_round(v[j]);
            a.y[(int64_t)m * a.ldy + n] = __float2bfloat16_rn(g / (1.f + __expf(-g)) * __bfloat162float(up[c + j]));
          }
        }
      }
    }
  } else {
  // part 2: every CTA of the cluster has seen its accumulator complete, so every
  // stage ring is free; push the fp32 rows to the CTAs (same pair position)
  // that own each 8-feature group
  __syncwarp();
  tc::cluster_sync_all();
  const int Cn = a.splits;
  const int rows_per_src = a.gmax * 8;
  const uint32_t red = smem_u32(smem);
  if (warp >= kEpiWarp0 && !dead && nkb > 0) {
    const int q = warp & 3;  // the TMEM lane quarter this warp may read
    const int f = q * 32 + lane;
    const int grp = f >> 3;
    const int owner = ((grp + 1) * Cn + 15) / 16 - 1;
    const int fl = (grp - owner * 16 / Cn) * 8 + (f & 7);  // row inside the owner's part
    const uint32_t dst =
        tc::map_to_rank(red + (uint32_t)(((split * rows_per_src + fl) * C::kPitch) * 4), (uint32_t)(2 * owner + member));
    const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
    for (int c = 0; c < MT; c += 32) {
      float v[32];
      tc::tmem_ld32(trow + c, v);
#pragma unroll
      for (int j = 0; j < 32; j += 4) tc::st_cluster_v4(dst + (uint32_t)(c + j) * 4, v[j], v[j + 1], v[j + 2], v[j + 3]);
    }
  }
  tc::fence_before();
  __syncwarp();
  tc::cluster_sync_all();
  if (G) {
    // gated with a K split: each CTA of split o now owns groups [g0, g0 + ng)
    // of its member's rows (gate in even CTAs, up in odd); the up owner sums
    // its parts, rounds them to bf16 and stores them behind the gate owner's
    // landing area; after the barrier the gate owner writes silu(g) * u
    const float* rf = reinterpret_cast<const float*>(smem);
    const int e = threadIdx.x - kEpiWarp0 * 32;
    const int g0 = split * 16 / Cn, ng = (split + 1) * 16 / Cn - g0;
    const int groups = ng * MT;
    const uint32_t up_off = (uint32_t)(Cn * rows_per_src * C::kPitch * 4);
    if (warp >= kEpiWarp0 && !dead && member == 1) {
      const uint32_t ub = tc::map_to_rank(red + up_off, rank & ~1u);
#pragma unroll 1
      for (int g = e; g < groups; g += 128) {
        const int ml = g % MT, fg = g / MT;
        if (m_tile * MT + ml >= a.M) continue;
#pragma unroll 1
        for (int j = 0; j < 8; ++j) {
          float acc = 0.f;
          for (int s2 = 0; s2 < Cn; ++s2) acc += rf[(s2 * rows_per_src + fg * 8 + j) * C::kPitch + ml];
          const bf16 h = __float2bfloat16_rn(acc);
          tc::st_cluster_b16(ub + (uint32_t)(((fg * 8 + j) * C::kUpPitch + ml) * 2),
                             *reinterpret_cast<const unsigned short*>(&h));
        }
      }
    }
    tc::fence_before();
    __syncwarp();
    tc::cluster_sync_all();
    if (warp >= kEpiWarp0 && !dead && member == 0) {
      const bf16* up = reinterpret_cast<const bf16*>(smem + up_off);
      const int nb = n0 + g0 * 8, m0 = m_tile * MT;
#pragma unroll 1
      for (int g = e; g < groups; g += 128) {
        const int ml = g % MT, fg = g / MT;
        const int m = m0 + ml;
        if (m >= a.M) continue;
        float y8[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float acc = 0.f;
          for (int s2 = 0; s2 < Cn; ++s2) acc += rf[(s2 * rows_per_src + fg * 8 + j) * C::kPitch + ml];
          const float gt = bf16_round(acc);
          y8[j] = gt / (1.f + __expf(-gt)) * __bfloat162float(up[(fg * 8 + j) * C::kUpPitch + ml]);
        }
        const int n = nb + fg * 8;
        if (n >= a.up_row0) continue;
        bf16* yr = a.y + (int64_t)m * a.ldy + n;
        if (a.vec_out && n + 8 <= a.up_row0) {
          uint4 pk;
          __nv_bfloat162* h2 = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
          for (int j = 0; j < 4; ++j) h2[j] = __floats2bfloat162_rn(y8[2 * j], y8[2 * j + 1]);
          *reinterpret_cast<uint4*>(yr) = pk;
        } else {
          for (int j = 0; j < 8 && n + j < a.up_row0; ++j) yr[j] = __float2bfloat16_rn(y8[j]);
        }
      }
    }
  }
  // part 3: this CTA owns feature groups [g0, g0 + ng) of its 128 rows
  if (!G && warp >= kEpiWarp0 && !dead) {
    const float* rf = reinterpret_cast<const float*>(smem);
    const int e = threadIdx.x - kEpiWarp0 * 32;
    const int g0 = split * 16 / Cn, ng = (split + 1) * 16 / Cn - g0;
    const int groups = ng * MT;
    const int nb = n0 + g0 * 8, m0 = m_tile * MT;
#pragma unroll 1
    for (int g = e; g < groups; g += 128) {
      const int ml = g % MT, fg = g / MT;
      const int m = m0 + ml;
      if (m >= a.M) continue;
      float acc[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
#pragma unroll 1
      for (int s = 0; s < Cn; ++s) {
        const float* p = rf + ((s * rows_per_src + fg * 8) * C::kPitch + ml);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] += p[j * C::kPitch];
      }
      const int n = nb + fg * 8;
      if (n >= a.N) continue;
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

  }  // not gated

  // TMEM reads are done in both CTAs of the pair before either frees the pair's allocation
  tc::fence_before();
  tc::cluster_sync_all();
  if (warp == 1) {
    tc::fence_after();
    tc::tmem_free_pair(tmem, C::kTmemCols);
  }
}

// ------------------------------------------------------------------ host side
int encode_rows(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
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

struct PairPlan {
  int mt, n_tiles, m_tiles, splits, kb_total, kb_per_split, ctas;
};

bool landing_fits(int mt, int splits, bool gated) {
  switch (mt) {
    case 64: return pair_landing_fits<64>(splits, gated);
    case 128: return pair_landing_fits<128>(splits, gated);
    default: return pair_landing_fits<256>(splits, gated);
  }
}

// Token tile: the smallest of 64 / 128 / 256 that holds the batch (256 beyond).
// K split (pairs per tile, 1..8, every part non-empty, the reduction inside
// the ring): the one with the fewest K-steps on the critical path, counting
// waves of one CTA per SM — ceil(2 x tiles x splits / SMs) x (ceil(K-steps /
// splits) + a reduction worth kReduceSteps K-steps when split); e.g. 96
// gate-up tiles: 3 splits, 4 waves x (22 + 4) steps, beat 2 waves x 64; ties
// go to the smaller split. splits_req > 0 asks for that split instead
// (reduced until valid).
constexpr int kReduceSteps = 4;

// gated: N is the output width I, a tile is 128 features (gate and up rows).
PairPlan make_pair_plan(int M, int N, int K, int splits_req, bool gated = false) {
  PairPlan p;
  p.mt = M <= 64 ? 64 : (M <= 128 ? 128 : 256);
  p.n_tiles = gated ? (N + kSlab - 1) / kSlab : (N + 2 * kSlab - 1) / (2 * kSlab);
  p.m_tiles = (M + p.mt - 1) / p.mt;
  p.kb_total = (K + kBK - 1) / kBK;
  const int tiles = p.n_tiles * p.m_tiles;
  auto valid = [&](int v) {
    if (v > p.kb_total) return false;
    const int per = (p.kb_total + v - 1) / v;
    return (v - 1) * per < p.kb_total && landing_fits(p.mt, v, gated);
  };
  int s = 1;
  if (splits_req > 0) {
    s = splits_req > kMaxSplits ? kMaxSplits : splits_req;
    while (s > 1 && !valid(s)) --s;
  } else {
    const int64_t nsm = device_sm_count();
    int64_t best = -1;
    for (int v = 1; v <= kMaxSplits; ++v) {
      if (v > 1 && !valid(v)) continue;
      const int64_t waves = (2 * (int64_t)tiles * v + nsm - 1) / nsm;
      const int64_t cost = waves * ((p.kb_total + v - 1) / v + (v > 1 ? kReduceSteps : 0));
      if (best < 0 || cost < best) {
        best = cost;
        s = v;
      }
    }
  }
  p.splits = s;
  p.kb_per_split = (p.kb_total + s - 1) / s;
  p.ctas = tiles * 2 * s;
  return p;
}

std::atomic<unsigned long long> g_attr_done{0};

template <int MT, bool G>
int launch_pair(const CUtensorMap& wmap, const CUtensorMap& xmap, const PairArgs& a, int ctas, cudaStream_t stream) {
  using C = PairCfg<MT>;
  int dev = 0;
  cudaGetDevice(&dev);
  // kernel attributes are set once per device (up to 8 cached; others every call)
  const unsigned long long bit =
      dev >= 0 && dev < 8 ? 1ull << (dev * 6 + (G ? 3 : 0) + (MT == 64 ? 0 : (MT == 128 ? 1 : 2))) : 0;
  if (!bit || !(g_attr_done.load() & bit)) {
    cudaError_t e = cudaFuncSetAttribute(gemm_pair_kernel<MT, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(gemm_pair_kernel<MT, G>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return cuda_status(e, "gemm pair kernel attributes");
    g_attr_done.fetch_or(bit);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = C::kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2 * a.splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, gemm_pair_kernel<MT, G>, wmap, xmap, a), "kvb_gemm_pair launch");
}

// y[M, n_out] = x w^T (gated: w = [gate | up] with n_out rows each, y = silu(x w_gate^T) * (x w_up^T)).
int run_pair(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy, int M, int n_out, int K,
             int splits, void* stream, bool gated, const char* name) {
  if (M < 0 || n_out <= 0 || K <= 0 || splits < 0 || splits > kMaxSplits || ldx < K || ldw < K || ldy < n_out)
    return set_error(kInvalid, "%s: bad sizes or leading dimensions", name);
  if (M == 0) return kOk;
  if (!x || !w || !y) return set_error(kInvalid, "%s: NULL pointer", name);
  if (((uintptr_t)x & 15) || ((uintptr_t)w & 15) || ldx % 8 || ldw % 8 || K % 8)
    return set_error(kInvalid, "%s: x/w rows must be 16-byte aligned (K, ldx, ldw multiples of 8)", name);
  const PairPlan p = make_pair_plan(M, n_out, K, splits, gated);
  CUtensorMap wmap, xmap;
  int rc = encode_rows(&wmap, w, (int64_t)n_out * (gated ? 2 : 1), K, ldw, kSlab);
  if (rc) return rc;
  rc = encode_rows(&xmap, x, M, K, ldx, p.mt / 2);
  if (rc) return rc;
  PairArgs a;
  a.y = (bf16*)y;
  a.ldy = ldy;
  a.M = M;
  a.N = n_out;
  a.n_tiles = p.n_tiles;
  a.m_tiles = p.m_tiles;
  a.splits = p.splits;
  a.kb_total = p.kb_total;
  a.kb_per_split = p.kb_per_split;
  a.gmax = (16 + p.splits - 1) / p.splits;
  // f32 D (bit 4), bf16 A and B (bits 7, 10), both K-major; N = MT (bits 17..22, N >> 3), M = 256 (bits 24..28, M >> 4)
  a.idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(p.mt >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
  a.vec_out = ((uintptr_t)y & 15) == 0 && ldy % 8 == 0;
  a.up_row0 = n_out;
  cudaStream_t st = (cudaStream_t)stream;
  if (gated) {
    switch (p.mt) {
      case 64: return launch_pair<64, true>(wmap, xmap, a, p.ctas, st);
      case 128: return launch_pair<128, true>(wmap, xmap, a, p.ctas, st);
      default: return launch_pair<256, true>(wmap, xmap, a, p.ctas, st);
    }
  }
  switch (p.mt) {
    case 64: return launch_pair<64, false>(wmap, xmap, a, p.ctas, st);
    case 128: return launch_pair<128, false>(wmap, xmap, a, p.ctas, st);
    default: return launch_pair<256, false>(wmap, xmap, a, p.ctas, st);
  }
}

}  // namespace
}  // namespace kvb

using namespace kvb;

extern "C" int kvb_gemm_pair_plan(int M, int N, int K, int splits, int gated, int* plan) {
  if (!plan || M <= 0 || N <= 0 || K <= 0 || splits < 0 || splits > kMaxSplits)
    return set_error(kInvalid, "kvb_gemm_pair_plan: bad sizes");
  const PairPlan p = make_pair_plan(M, N, K, splits, gated != 0);
  plan[0] = p.mt;
  plan[1] = p.splits;
  plan[2] = p.n_tiles * p.m_tiles;
  plan[3] = p.ctas;
  return kOk;
}

extern "C" int kvb_gemm_pair_bf16(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy, int M,
                                  int N, int K, int splits, void* stream) {
  return run_pair(x, ldx, w, ldw, y, ldy, M, N, K, splits, stream, false, "kvb_gemm_pair_bf16");
}

extern "C" int kvb_gemm_pair_silu_bf16(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy,
                                       int M, int inter, int K, int splits, void* stream) {
  return run_pair(x, ldx, w, ldw, y, ldy, M, inter, K, splits, stream, true, "kvb_gemm_pair_silu_bf16");
}
