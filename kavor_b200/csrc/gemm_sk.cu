// Decode-batch GEMM on CTA pairs with a stream-K schedule:
// Y[M, N] = X[M, K] W[N, K]^T (F.linear of linear.py:50,73,157 and
// embed_head.py:61), fp32 accumulation in TMEM, bf16 output; and the gate-up
// projection fused with SiluAndMul (linear.py:76-93 + activation.py:8-11).
//
// At decode (M <= 256 tokens) a projection streams its whole weight once and
// multiplies every weight byte by the whole batch, which puts it at the ridge
// of the B200 (256 FLOP per weight byte). The kernel is built so that every
// SM streams weights at its share of HBM bandwidth for the whole launch:
//
// * pairs: two CTAs of a 2-CTA cluster issue one tcgen05.mma.cta_group::2 of
//   M = 256 weight rows (128 in each CTA's shared memory) x N = MT tokens
//   (MT/2 token rows staged in each CTA) x K = 16. A stage is KC chunks of
//   64 K: one 3-D TMA load of the CTA's 128 weight rows x KC chunks (KC x 16
//   KB) and one of its MT/2 token rows (an SM streams one multi-chunk load at
//   about twice the rate of separate 16 KB boxes). Both CTAs' loads (no
//   multicast) complete on the even CTA's barrier; the MMA thread's commits
//   release each stage in both CTAs;
// * stream-K: the grid is one wave of persistent pairs (2-CTA clusters always
//   fit); the (tile, K step) iterations of the whole GEMM are dealt to the
//   pairs in equal contiguous ranges, so every pair streams the same number
//   of weight bytes whatever the tile count. A range cuts tiles into
//   segments: a tile covered by one segment is written directly; otherwise
//   the segment holding the tile's first K steps (the last segment of its
//   pair) owns it, and each later segment (the first segment of a later pair)
//   leaves an fp32 partial in the caller's workspace and raises a flag; the
//   owner adds the partials in K order (deterministic) and writes bf16;
// * two TMEM accumulators: the MMAs of a pair's next segment run while the
//   epilogue warps drain the previous one;
// * warp 0 issues TMA, warp 1 holds the pair's TMEM and (even CTA) issues the
//   MMAs, warps 2..5 drain TMEM (one lane quarter each) through a per-warp
//   shared-memory transpose into 16-byte row stores.
//
// Gated form: a pair tile is 128 output features; each CTA's 128 weight rows
// are 64 gate rows [n, n + 64) and the matching 64 up rows [I + n, I + n + 64)
// of the [gate | up] weight (a 4-D load whose third coordinate steps from the
// gate to the up half; weight layout unchanged), so gate
// and up of a feature sit in the same CTA's TMEM (lanes r and 64 + r); the up
// warps hand bf16(up) to the gate warps through shared memory, which write
// bf16(silu(bf16(gate)) * up) — the reference's rounding points.
//
// Workspace (caller-owned, zeroed once when allocated): two hand-off flags
// per pair, then per pair one partial slot of 2 x 128 x MT fp32. Every flag is back at zero when a
// launch completes normally; after a device error (a wait gave up) the
// workspace must be zeroed again. Calls that share a workspace must be
// stream-ordered. Every wait is bounded (kSpinCycles).
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>

#include "common.cuh"
#include "tcgen05.cuh"
#include "../../include/kavor_b200.h"

KVB_DEFINE_ERROR_WORD(gemm_sk)

namespace kvb {
namespace {

constexpr int kBK = 64;          // K elements per chunk (one 128-byte swizzle row)
constexpr int kRows = 128;       // weight rows per CTA (half of the pair's UMMA M)
constexpr int kThreads = 192;    // 6 warps
constexpr int kEpiWarp0 = 2;
constexpr int kEpiThreads = 128;
constexpr int kMaxPairs = 128;

struct SkArgs {
  bf16* y;
  int64_t ldy;
  float* partial;     // [pairs][2][128][MT] fp32
  unsigned* flags;    // [pairs][2]
  int M, N;           // N: output features (gated: the intermediate size I)
  int up_row0;        // gated: first weight row of the up half (= I)
  int m_tiles;
  int kb;             // K steps of 64
  long long iters;    // tiles x kb
  int pairs;
  uint32_t idesc;
  int vec_out;
};

template <int MT, bool G>
struct SkCfg {
  static constexpr int kHalf = MT / 2;                    // token rows each CTA stages
  static constexpr int kKC = MT >= 128 ? 2 : 3;           // 64-wide K chunks per stage
  static constexpr int kAChunk = kRows * kBK * 2;         // 16 KB of weight per chunk
  static constexpr int kBChunk = kHalf * kBK * 2;
  static constexpr int kABytes = kKC * kAChunk;
  static constexpr int kBBytes = kKC * kBChunk;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kRing = 196 * 1024;
  static constexpr int kStagesRaw = kRing / kStageBytes;
  static constexpr int kStages = kStagesRaw > 8 ? 8 : kStagesRaw;
  static constexpr int kChunk = MT < 32 ? MT : 32;        // tokens per TMEM load
  static constexpr int kTmemCols = 2 * MT < 32 ? 32 : 2 * MT;
  static constexpr int kXpose = 4 * 32 * kChunk * 2;      // per-warp bf16 transpose tiles
  static constexpr int kUp = G ? 2 * 64 * kChunk * 2 : 0; // gated: two chunks of up values, 64 features
  static constexpr int kSmem = kStages * kStageBytes + kXpose + kUp + 1024;
  static_assert(MT == 16 || MT == 32 || MT == 64 || MT == 128 || MT == 256, "token tile");
  static_assert(kStages >= 3, "stage ring depth");
  static_assert(kSmem <= 227 * 1024, "dynamic shared memory of one CTA");
  static_assert(kTmemCols <= 512, "TMEM columns of one SM");
  static_assert(kAChunk % 1024 == 0 && kBChunk % 1024 == 0, "swizzle atoms stay 1024-byte aligned");
};

// Pair p's iterations: [p * iters / pairs, (p + 1) * iters / pairs) (the host
// keeps pairs * iters below 2^32, so the division is 32-bit).
__device__ __forceinline__ long long range_lo(const SkArgs& a, int p) {
  return (long long)((uint32_t)p * (uint32_t)a.iters / (uint32_t)a.pairs);
}

__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(unsigned* p, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// AND of `pred` over the `n` threads of named barrier `id` (all of them get it).
__device__ __forceinline__ bool bar_and(int id, int n, bool pred) {
  int r;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\tsetp.ne.s32 pi, %1, 0;\n\tbar.red.and.pred po, %2, %3, pi;\n\t"
      "selp.s32 %0, 1, 0, po;\n\t}"
      : "=r"(r)
      : "r"((int)pred), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}

// Bounded wait on an mbarrier phase that gives up at once when `dead` is set.
__device__ __forceinline__ bool sk_wait(uint32_t bar, uint32_t parity, volatile int* dead) {
  if (mbar_try_wait(bar, parity)) return true;
  if (*dead) return false;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (*dead) return false;
    if (clock64() - t0 > kSpinCycles) {
      atomicOr(&g_err_gemm_sk, (unsigned)kErrTimeout);
      *dead = 1;
      return false;
    }
  }
  return true;
}

// Segment walker: the (tile, k0, k1) pieces of pair p's range, in order.
struct Seg {
  int tile, k0, k1;
};
struct SegIter {
  long long it, hi;
  int kb;
  __device__ bool next(Seg& s) {
    if (it >= hi) return false;
    s.tile = (int)(it / kb);
    s.k0 = (int)(it - (long long)s.tile * kb);
    const long long left = hi - it;
    s.k1 = left < (long long)(kb - s.k0) ? s.k0 + (int)left : kb;
    it += s.k1 - s.k0;
    return true;
  }
};

template <int MT, bool G>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_sk_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                   const __grid_constant__ SkArgs a) {
  using C = SkCfg<MT, G>;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[S];
  __shared__ __align__(8) uint64_t empty_bar[S];
  __shared__ __align__(8) uint64_t tfull_bar[2];
  __shared__ __align__(8) uint64_t tempty_bar[2];
  __shared__ __align__(8) uint64_t red_bar;
  __shared__ uint32_t tmem_base_s;
  __shared__ int dead_s;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* xpose = smem + S * C::kStageBytes;
  bf16* upbuf = reinterpret_cast<bf16*>(xpose + C::kXpose);
  volatile int* dead = &dead_s;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = tc::cluster_rank();
  const int member = (int)(rank & 1u);
  const int pair = (int)blockIdx.x >> 1;
  const uint32_t leader = rank & ~1u;
  const uint16_t pair_mask = (uint16_t)(3u << leader);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&tfull_bar[b]), 1);
      mbar_init(smem_u32(&tempty_bar[b]), 2 * (kEpiThreads / 32));  // 4 epilogue warps x 2 CTAs
    }
    mbar_init(smem_u32(&red_bar), 1);
    dead_s = 0;
    fence_barrier_init();
  }
  if (warp == 1) tc::tmem_alloc_pair(smem_u32(&tmem_base_s), C::kTmemCols);
  tc::fence_before();
  tc::cluster_sync_all();  // both CTAs' barriers and the pair's TMEM exist before either signals the other's
  tc::fence_after();
  kernel_entry();          // token rows, outputs and the workspace belong to the kernels before this one
  const uint32_t tmem = tmem_base_s;
  const long long lo = range_lo(a, pair), hi = range_lo(a, pair + 1);

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      prefetch_tensormap(&wmap);
      prefetch_tensormap(&xmap);
      // one thread, so the per-stage work is kept to a few dependent instructions:
      // running slot / phase counters, shared-memory addresses advanced by a constant
      SegIter segs{lo, hi, a.kb};
      Seg sg;
      uint32_t issued = 0, phase = 0;
      int s = 0;
      const uint32_t ring0 = smem_u32(smem), full0 = smem_u32(&full_bar[0]), empty0 = smem_u32(&empty_bar[0]);
      const uint32_t full0_leader = tc::map_to_rank(full0, leader);
      bool ok = true;
      while (ok && segs.next(sg)) {
        const int n_tile = sg.tile / a.m_tiles, m_tile = sg.tile - n_tile * a.m_tiles;
        const int wrow = G ? n_tile * 128 + member * 64 : n_tile * 256 + member * kRows;  // gated: within a half
        const int xrow = m_tile * MT + member * C::kHalf;
        for (int k = sg.k0; k < sg.k1; ++k) {
          if (issued >= (uint32_t)S && !sk_wait(empty0 + 8 * s, phase ^ 1u, dead)) {
            ok = false;
            break;
          }
          const uint32_t sa = ring0 + (uint32_t)(s * C::kStageBytes);
          const uint32_t fl = full0_leader + 8 * s;
          if (member == 0) mbar_arrive_expect_tx(full0 + 8 * s, 2 * C::kStageBytes);
          // [chunk][128 weight rows][64 K] (gated: each chunk 64 gate rows, then the same features' up rows)
          if (G) tc::tma_load_4d_pair(sa, &wmap, 0, wrow, 0, k * C::kKC, fl);
          else tc::tma_load_3d_pair(sa, &wmap, 0, wrow, k * C::kKC, fl);
          tc::tma_load_3d_pair(sa + C::kABytes, &xmap, 0, xrow, k * C::kKC, fl);
          ++issued;
          if (++s == S) {
            s = 0;
            phase ^= 1u;
          }
        }
      }
      // before the CTA exits: the loads of the last stages have landed (leader's
      // barriers) and, after a normal run, the MMA thread's releases of them have
      // arrived on this CTA's barriers; one overall bound
      const long long t0 = clock64();
      for (uint32_t i = issued > (uint32_t)S ? issued - S : 0; i < issued; ++i) {
        bool late = false;
        if (member == 0)
          while (!late && !mbar_try_wait(smem_u32(&full_bar[i % S]), (i / S) & 1)) late = clock64() - t0 > kSpinCycles;
        while (!late && !*dead && !mbar_try_wait(smem_u32(&empty_bar[i % S]), (i / S) & 1))
          late = clock64() - t0 > kSpinCycles;
        if (late) break;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (even CTA)
    if (lane == 0 && member == 0) {
      SegIter segs{lo, hi, a.kb};
      Seg sg;
      uint32_t j = 0, phase = 0;
      int s = 0;
      const uint32_t full0 = smem_u32(&full_bar[0]), empty0 = smem_u32(&empty_bar[0]);
      // descriptors of stage 0; a stage's are these plus its byte offset / 16 (the address field)
      const uint64_t da0 = tc::smem_desc_sw128(smem_u32(smem)), db0 = tc::smem_desc_sw128(smem_u32(smem) + C::kABytes);
      bool ok = true;
      while (ok && segs.next(sg)) {
        const int b = (int)(j & 1);
        if (j >= 2 && !sk_wait(smem_u32(&tempty_bar[b]), ((j >> 1) - 1) & 1, dead)) break;
        tc::fence_after();
        const uint32_t d = tmem + (uint32_t)(b * MT);
        for (int k = sg.k0; k < sg.k1; ++k) {
          if (!sk_wait(full0 + 8 * s, phase, dead)) {
            ok = false;
            break;
          }
          tc::fence_after();
          const uint64_t off = (uint64_t)(s * (C::kStageBytes >> 4));
          const uint64_t da = da0 + off, db = db0 + off;
          tc::umma_pair_bf16(d, da, db, a.idesc, k > sg.k0 ? 1u : 0u);
#pragma unroll
          for (int kk = 1; kk < 4 * C::kKC; ++kk) {
            // chunk kk / 4 sits a whole chunk further on; inside a chunk +32 B along K = +2
            const uint64_t ca = (uint64_t)((kk >> 2) * (C::kAChunk >> 4) + 2 * (kk & 3));
            const uint64_t cb = (uint64_t)((kk >> 2) * (C::kBChunk >> 4) + 2 * (kk & 3));
            tc::umma_pair_bf16(d, da + ca, db + cb, a.idesc, 1u);
          }
          tc::umma_commit_pair(empty0 + 8 * s, pair_mask);
          if (++s == S) {
            s = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc::umma_commit_pair(smem_u32(&tfull_bar[b]), pair_mask);
        ++j;
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;                   // TMEM lane quarter of this warp
    const int r = q * 32 + lane;              // this thread's weight row in the CTA (TMEM lane)
    const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16);
    bf16* xp = reinterpret_cast<bf16*>(xpose) + (warp - kEpiWarp0) * 32 * C::kChunk;
    const int e = threadIdx.x - kEpiWarp0 * 32;
    const uint32_t tempty_leader0 = tc::map_to_rank(smem_u32(&tempty_bar[0]), leader);
    const float* ring = reinterpret_cast<const float*>(smem);
    uint32_t red_uses = 0;  // completed phases of red_bar

    // bf16 rows of one 32-token (16 for MT = 16) chunk: lane = feature, through the
    // per-warp transpose into 16-byte stores of 8 features per token; gated: the up
    // rows hand bf16(up) to the gate rows of the same features first
    auto emit = [&](float* v, int n_tile, int m0, int c) {
      int nbase;
      bool writer = true;
      if constexpr (G) {
        bf16* ub = upbuf + ((c / C::kChunk) & 1) * 64 * C::kChunk;  // [token][64 features], two chunks
        if (q >= 2) {
#pragma unroll
          for (int jj = 0; jj < C::kChunk; ++jj) ub[jj * 64 + (r - 64)] = __float2bfloat16_rn(v[jj]);
        }
        named_bar_sync(2, kEpiThreads);
        if (q < 2) {
#pragma unroll
          for (int jj = 0; jj < C::kChunk; ++jj) {
            const float g = bf16_round(v[jj]);
            v[jj] = g / (1.f + __expf(-g)) * __bfloat162float(ub[jj * 64 + r]);
          }
        }
        writer = q < 2;
        nbase = n_tile * 128 + member * 64 + q * 32;
      } else {
        nbase = n_tile * 256 + member * kRows + q * 32;
      }
      if (!writer) return;
#pragma unroll
      for (int jj = 0; jj < C::kChunk; ++jj) xp[jj * 32 + lane] = __float2bfloat16_rn(v[jj]);
      __syncwarp();
#pragma unroll
      for (int it = 0; it < C::kChunk * 4 / 32; ++it) {
        const int idx = it * 32 + lane;
        const int tok = idx >> 2, part = idx & 3;
        const int m = m0 + c + tok, n = nbase + part * 8;
        if (m < a.M && n < a.N) {
          const uint4 pk = *reinterpret_cast<const uint4*>(xp + tok * 32 + part * 8);
          bf16* yr = a.y + (int64_t)m * a.ldy + n;
          if (a.vec_out && n + 8 <= a.N) {
            *reinterpret_cast<uint4*>(yr) = pk;
          } else {
            const bf16* h = reinterpret_cast<const bf16*>(&pk);
            for (int t = 0; t < 8 && n + t < a.N; ++t) yr[t] = h[t];
          }
        }
      }
      __syncwarp();
    };
    auto tmem_ld = [&](uint32_t addr, float* v) {
      if constexpr (C::kChunk == 32) tc::tmem_ld32(addr, v);
      else tc::tmem_ld16(addr, v);
    };

    SegIter segs{lo, hi, a.kb};
    Seg sg;
    uint32_t j = 0;
    while (segs.next(sg)) {
      const int b = (int)(j & 1);
      const bool have = sk_wait(smem_u32(&tfull_bar[b]), (j >> 1) & 1, dead);
      // one decision for the four warps (named-barrier participation never depends on a per-warp view)
      bool ok = bar_and(1, kEpiThreads, have && !*dead);
      tc::fence_after();
      const int n_tile = sg.tile / a.m_tiles, m_tile = sg.tile - n_tile * a.m_tiles;
      const int m0 = m_tile * MT;
      const uint32_t tb = tq + (uint32_t)(b * MT);
      const bool contributor = sg.k0 > 0;
      const bool owner = sg.k0 == 0 && sg.k1 < a.kb;
      if (contributor) {
        // fp32 partial, token-major ([MT][128 rows]: a warp's stores and the owner's
        // shared-memory reads are consecutive), then the flag
        float* slot = a.partial + ((size_t)pair * 2 + member) * kRows * MT;
        if (ok) {
#pragma unroll 1
          for (int c = 0; c < MT; c += C::kChunk) {
            float v[C::kChunk];
            tmem_ld(tb + c, v);
#pragma unroll
            for (int jj = 0; jj < C::kChunk; ++jj) slot[(size_t)(c + jj) * kRows + r] = v[jj];
          }
        }
        tc::fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(tempty_leader0 + (uint32_t)(b * 8));
        named_bar_sync(1, kEpiThreads);  // every row of the partial is written
        if (ok && e == 0) {
          __threadfence();
          st_release_gpu(a.flags + 2 * pair + member, 1u);
        }
      } else if (!owner) {
        // the whole tile in one segment
        if (ok) {
#pragma unroll 1
          for (int c = 0; c < MT; c += C::kChunk) {
            float v[C::kChunk];
            tmem_ld(tb + c, v);
            emit(v, n_tile, m0, c);
          }
        }
        tc::fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(tempty_leader0 + (uint32_t)(b * 8));
      } else {
        // owner: the pair's last segment, so the stage ring is idle; the later
        // segments' partials come in by bulk copies, as many per round as fit,
        // and are added in K order (sums kept in TMEM between rounds)
        int c_last = pair;
        const long long tile_end = (long long)(sg.tile + 1) * a.kb;
        while (c_last + 1 < a.pairs && range_lo(a, c_last + 1) < tile_end) ++c_last;
        if (ok && e == 0) {
          for (int cc = pair + 1; cc <= c_last && !*dead; ++cc) {
            const unsigned* f = a.flags + 2 * cc + member;
            const long long t0 = clock64();
            while (ld_acquire_gpu(f) != 1u) {
              if (clock64() - t0 > kSpinCycles) {
                atomicOr(&g_err_gemm_sk, (unsigned)kErrTimeout);
                *dead = 1;
                break;
              }
            }
          }
          asm volatile("fence.proxy.async.global;" ::: "memory");  // the bulk copies read what the flags published
        }
        ok = bar_and(1, kEpiThreads, ok && !*dead);
        constexpr uint32_t kPart = (uint32_t)kRows * MT * 4;
        constexpr int kFitRaw = (S * C::kStageBytes) / (int)kPart;
        constexpr int kFit = kFitRaw < 1 ? 1 : kFitRaw;
        static_assert(kFitRaw >= 1, "one partial fits the stage ring");
        int g0 = pair + 1;
        do {
          const int n = g0 <= c_last ? min(kFit, c_last - g0 + 1) : 0;
          const bool last = g0 + n > c_last;
          if (ok && n > 0) {
            if (e == 0) {
              asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // earlier ring reads before the copies
              const uint32_t rb = smem_u32(&red_bar);
              mbar_arrive_expect_tx(rb, (uint32_t)n * kPart);
              for (int i = 0; i < n; ++i)
                tc::bulk_load(smem_u32(smem) + (uint32_t)i * kPart,
                              a.partial + ((size_t)(g0 + i) * 2 + member) * kRows * MT, kPart, rb);
            }
            const bool got = sk_wait(smem_u32(&red_bar), red_uses & 1, dead);
            ok = bar_and(1, kEpiThreads, got);
            ++red_uses;
          }
          if (ok) {
#pragma unroll 1
            for (int c = 0; c < MT; c += C::kChunk) {
              float v[C::kChunk];
              tmem_ld(tb + c, v);
              for (int i = 0; i < n; ++i) {
                const float* pr = ring + (size_t)i * kRows * MT + (size_t)c * kRows + r;
#pragma unroll
                for (int jj = 0; jj < C::kChunk; ++jj) v[jj] += pr[jj * kRows];
              }
              if (last) {
                emit(v, n_tile, m0, c);
              } else if constexpr (C::kChunk == 32) {
                tc::tmem_st32(tb + c, v);
              } else {
                tc::tmem_st16(tb + c, v);
              }
            }
          }
          named_bar_sync(1, kEpiThreads);  // the ring is read before the next round's copies land
          g0 += n;
          if (n == 0) break;
        } while (g0 <= c_last);
        tc::fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(tempty_leader0 + (uint32_t)(b * 8));
        if (ok && e == 0)
          for (int cc = pair + 1; cc <= c_last; ++cc) a.flags[2 * cc + member] = 0u;
      }
      ++j;
    }
  }

  // TMEM reads and MMAs are done in both CTAs of the pair before either frees the allocation
  tc::fence_before();
  __syncthreads();
  tc::cluster_sync_all();
  if (warp == 1) {
    tc::fence_after();
    tc::tmem_free_pair(tmem, C::kTmemCols);
  }
}

// ------------------------------------------------------------------ host side
// [chunks of 64 K][rows][64 K] views: a 3-D map {64, rows, K / 64} whose box
// is {64, box_rows, kc}, 128-byte swizzle; gated, a 4-D map {64, 64-row
// blocks... } whose third coordinate steps from the gate half to the up half.
int encode_chunks(CUtensorMap* map, const void* base, int64_t rows, int64_t K, int64_t ld, int box_rows, int kc,
                  int64_t half_rows) {
  auto enc = tensor_map_encoder();
  if (!enc) return set_error(kNoEncoder, "cuTensorMapEncodeTiled is not available from the driver");
  CUresult r;
  if (half_rows == 0) {
    const cuuint64_t dims[3] = {(cuuint64_t)kBK, (cuuint64_t)rows, (cuuint64_t)(K / kBK)};
    const cuuint64_t strides[2] = {(cuuint64_t)ld * 2, (cuuint64_t)kBK * 2};
    const cuuint32_t box[3] = {(cuuint32_t)kBK, (cuuint32_t)box_rows, (cuuint32_t)kc};
    const cuuint32_t estr[3] = {1, 1, 1};
    r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    // {64 K, rows of one half, 2 halves (gate, up), K / 64}; box {64, 64, 2, kc}
    const cuuint64_t dims[4] = {(cuuint64_t)kBK, (cuuint64_t)half_rows, 2, (cuuint64_t)(K / kBK)};
    const cuuint64_t strides[3] = {(cuuint64_t)ld * 2, (cuuint64_t)half_rows * ld * 2, (cuuint64_t)kBK * 2};
    const cuuint32_t box[4] = {(cuuint32_t)kBK, (cuuint32_t)box_rows, 2, (cuuint32_t)kc};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  if (r != CUDA_SUCCESS) return set_error(kEncode, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
  return kOk;
}

struct SkPlan {
  int mt, n_tiles, m_tiles, kb, pairs;
  long long iters;
};

int token_tile(int M) {
  int mt = 16;
  while (mt < M && mt < 256) mt <<= 1;
  return mt;
}

int sk_stages(int mt) {
  switch (mt) {
    case 16: return SkCfg<16, false>::kStages;
    case 32: return SkCfg<32, false>::kStages;
    case 64: return SkCfg<64, false>::kStages;
    case 128: return SkCfg<128, false>::kStages;
    default: return SkCfg<256, false>::kStages;
  }
}
int sk_kc(int mt) { return mt >= 128 ? SkCfg<256, false>::kKC : SkCfg<16, false>::kKC; }

// Pairs: one wave (at most SMs / 2, and no more than fit together), and the
// count with the smallest modelled time. A pair's range of K steps runs at
// the slowest of: the HBM bandwidth shared by the streaming SMs, one SM's
// own load rate (about 110 GB/s for these multi-chunk loads) and the MMA rate
// (64-wide K chunk x 4 MMAs of max(59, MT / 2) cycles). A tile cut into
// pieces costs its owner the reading of the other pieces' fp32 partials and a
// hand-off latency. Ties go to more pairs.
SkPlan plan_for_tile(int M, int N, int K, bool gated, int mt, int max_pairs, double* cost) {
  SkPlan p;
  p.mt = mt;
  p.n_tiles = gated ? (N + 127) / 128 : (N + 255) / 256;
  p.m_tiles = (M + p.mt - 1) / p.mt;
  const int kc = sk_kc(p.mt);
  p.kb = (K / kBK + kc - 1) / kc;
  p.iters = (long long)p.n_tiles * p.m_tiles * p.kb;
  // every m-tile streams its n-tile's weights again (from HBM: the pieces of
  // one n-tile's m-tiles do not run close enough together to meet in L2)
  const double hbm = 6.8e12, sm_rate = 110e9, clk = 1.8e9;
  const double stage_w = 16384.0 * kc;
  const double t_mma = kc * 4 * std::max(59.0, p.mt / 2.0) / clk;
  // a cut tile: the contributors write their fp32 partials while their SM
  // streams the next segment, the owner reads them back (about 40 GB/s per
  // SM end to end, measured), plus the flag hand-off
  const double partial = (double)kRows * p.mt * 4, l2_rate = 40e9, handoff = 2e-6;
  const double t_epi = (double)kRows * p.mt * 2 / 40e9;  // the last tile's drain (bf16 rows out)
  double best = -1;
  p.pairs = 1;
  for (int P = (int)std::min<long long>(max_pairs, p.iters); P >= 1; --P) {
    const long long per = (p.iters + P - 1) / P;
    const double rate = std::min(sm_rate, hbm / (2.0 * P));
    const double t_stage = std::max(stage_w / rate, t_mma);
    const long long pieces = per >= p.kb ? (p.iters % P ? 2 : 1) : (p.kb + per - 1) / per + 1;
    const double t = per * t_stage + t_epi + (pieces > 1 ? handoff + (pieces - 1) * partial / l2_rate : 0.0);
    if (best < 0 || t < best * 0.99) {
      best = t;
      p.pairs = P;
    }
  }
  *cost = best;
  return p;
}

// Process-wide plan override for tuning sweeps (kvb_gemm_sk_set_plan):
// token tile and pair count, 0 = the model's choice.
std::atomic<int> g_sk_force_mt{0}, g_sk_force_pairs{0};

SkPlan make_sk_plan(int M, int N, int K, bool gated, int coresident = 0) {
  int max_pairs = std::min(kMaxPairs, device_sm_count() / 2);
  if (coresident > 0) max_pairs = std::min(max_pairs, coresident);
  double c1 = 0, c2 = 0;
  const int mt = token_tile(M);
  const int fmt = g_sk_force_mt.load(), fpairs = g_sk_force_pairs.load();
  if (fmt > 0 || fpairs > 0) {
    SkPlan p = plan_for_tile(M, N, K, gated, fmt > 0 && fmt <= mt ? fmt : mt, max_pairs, &c1);
    if (fpairs > 0) p.pairs = (int)std::min<long long>(std::min(fpairs, max_pairs), p.iters);
    return p;
  }
  SkPlan p = plan_for_tile(M, N, K, gated, mt, max_pairs, &c1);
  if (mt == 256 && M <= 256) {  // two 128-token tiles: half the partials and the drain, a deeper ring
    SkPlan q = plan_for_tile(M, N, K, gated, 128, max_pairs, &c2);
    if (c2 < c1) p = q;
  }
  return p;
}

// Workspace: the hand-off flags of every pair at a fixed place (so no plan's
// partials ever cover another plan's flags), then the partial slots.
constexpr size_t kFlagBytes = (size_t)kMaxPairs * 2 * sizeof(unsigned);
static_assert(kFlagBytes % 256 == 0, "partials start 256-byte aligned");

size_t sk_workspace_bytes(const SkPlan& p) {
  return kFlagBytes + (size_t)p.pairs * 2 * kRows * p.mt * sizeof(float);
}

// Pairs of this kernel variant that are resident together on the current
// device (the stream-K owners wait for later pairs, so the grid must be one
// wave); set up once per device and variant: the dynamic shared-memory limit
// and the occupancy query for 2-CTA clusters.
std::atomic<int> g_sk_pairs[8][10];

template <int MT, bool G>
int sk_coresident(int* out) {
  using C = SkCfg<MT, G>;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "gemm_sk: cudaGetDevice");
  const int variant = (G ? 5 : 0) + (MT == 16 ? 0 : MT == 32 ? 1 : MT == 64 ? 2 : MT == 128 ? 3 : 4);
  std::atomic<int>* slot = dev >= 0 && dev < 8 ? &g_sk_pairs[dev][variant] : nullptr;
  if (slot && slot->load() > 0) {
    *out = slot->load();
    return kOk;
  }
  e = cudaFuncSetAttribute(gemm_sk_kernel<MT, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
  if (e != cudaSuccess) return cuda_status(e, "gemm_sk kernel attributes");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * kMaxPairs, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = C::kSmem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  e = cudaOccupancyMaxActiveClusters(&clusters, gemm_sk_kernel<MT, G>, &cfg);
  if (e != cudaSuccess) return cuda_status(e, "gemm_sk: cudaOccupancyMaxActiveClusters");
  if (clusters <= 0) return set_error(kUnsupported, "gemm_sk: no 2-CTA cluster of this kernel fits on the device");
  if (slot) slot->store(clusters);
  *out = clusters;
  return kOk;
}

int sk_coresident_for(int mt, bool gated, int* out) {
#define KVB_SK_CASE(MTV) \
  case MTV:              \
    return gated ? sk_coresident<MTV, true>(out) : sk_coresident<MTV, false>(out);
  switch (mt) {
    KVB_SK_CASE(16)
    KVB_SK_CASE(32)
    KVB_SK_CASE(64)
    KVB_SK_CASE(128)
    KVB_SK_CASE(256)
  }
#undef KVB_SK_CASE
  return set_error(kUnsupported, "gemm_sk: token tile %d", mt);
}

template <int MT, bool G>
int launch_sk(const CUtensorMap& wmap, const CUtensorMap& xmap, const SkArgs& a, cudaStream_t stream) {
  using C = SkCfg<MT, G>;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * a.pairs, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = C::kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, gemm_sk_kernel<MT, G>, wmap, xmap, a), "kvb_gemm_sk launch");
}

int run_sk(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy, int M, int n_out, int K,
           void* workspace, size_t ws_bytes, void* stream, bool gated, const char* name) {
  if (M < 0 || n_out <= 0 || K <= 0 || ldx < K || ldw < K || ldy < n_out)
    return set_error(kInvalid, "%s: bad sizes or leading dimensions", name);
  if (M == 0) return kOk;
  if (!x || !w || !y) return set_error(kInvalid, "%s: NULL pointer", name);
  if (((uintptr_t)x & 15) || ((uintptr_t)w & 15) || ldx % 8 || ldw % 8)
    return set_error(kInvalid, "%s: x/w rows must be 16-byte aligned (ldx, ldw multiples of 8)", name);
  if (K % kBK) return set_error(kUnsupported, "%s: K must be a multiple of 64 (got %d)", name, K);
  if ((long long)((M + 15) / 16) * ((n_out + 127) / 128) * (K / kBK) * kMaxPairs >= (1ll << 32))
    return set_error(kUnsupported, "%s: shape too large for the stream-K schedule", name);
  if (!workspace) return set_error(kWorkspace, "%s: no workspace given (kvb_gemm_sk_workspace_size)", name);
  if ((uintptr_t)workspace & 255) return set_error(kInvalid, "%s: workspace must be 256-byte aligned", name);
  // 2-CTA clusters of every variant fit the same way (one CTA per SM): the
  // largest token tile's count bounds them all
  int coresident = 0;
  int rc = sk_coresident_for(token_tile(M), gated, &coresident);
  if (rc) return rc;
  const SkPlan p = make_sk_plan(M, n_out, K, gated, coresident);
  if (p.mt != token_tile(M)) {  // the variant the plan chose gets its shared-memory limit too
    int other = 0;
    rc = sk_coresident_for(p.mt, gated, &other);
    if (rc) return rc;
  }
  const size_t need = sk_workspace_bytes(p);
  if (ws_bytes < need)
    return set_error(kWorkspace, "%s: workspace of %zu bytes given, %zu needed (zeroed once when allocated)", name,
                     ws_bytes, need);
  CUtensorMap wmap, xmap;
  const int kc = sk_kc(p.mt);
  rc = gated ? encode_chunks(&wmap, w, 0, K, ldw, 64, kc, n_out) : encode_chunks(&wmap, w, n_out, K, ldw, kRows, kc, 0);
  if (rc) return rc;
  rc = encode_chunks(&xmap, x, M, K, ldx, p.mt / 2, kc, 0);
  if (rc) return rc;
  SkArgs a;
  a.y = (bf16*)y;
  a.ldy = ldy;
  a.flags = (unsigned*)workspace;
  a.partial = (float*)((uint8_t*)workspace + kFlagBytes);
  a.M = M;
  a.N = n_out;
  a.up_row0 = n_out;
  a.m_tiles = p.m_tiles;
  a.kb = p.kb;
  a.iters = p.iters;
  a.pairs = p.pairs;
  // f32 D (bit 4), bf16 A and B (bits 7, 10), both K-major; N = MT (bits 17..22, N >> 3); M = 256 (bits 24..28, M >> 4)
  a.idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(p.mt >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
  a.vec_out = ((uintptr_t)y & 15) == 0 && ldy % 8 == 0;
  cudaStream_t st = (cudaStream_t)stream;
#define KVB_SK_CASE(MTV)                                                                   \
  case MTV:                                                                                \
    return gated ? launch_sk<MTV, true>(wmap, xmap, a, st) : launch_sk<MTV, false>(wmap, xmap, a, st);
  switch (p.mt) {
    KVB_SK_CASE(16)
    KVB_SK_CASE(32)
    KVB_SK_CASE(64)
    KVB_SK_CASE(128)
    KVB_SK_CASE(256)
  }
#undef KVB_SK_CASE
  return set_error(kUnsupported, "%s: token tile %d", name, p.mt);
}

}  // namespace
}  // namespace kvb

using namespace kvb;

extern "C" int kvb_gemm_sk_plan(int M, int N, int K, int gated, int* plan) {
  if (!plan || M <= 0 || N <= 0 || K <= 0) return set_error(kInvalid, "kvb_gemm_sk_plan: bad sizes");
  const SkPlan p = make_sk_plan(M, N, K, gated != 0);
  plan[0] = p.mt;
  plan[1] = p.n_tiles * p.m_tiles;
  plan[2] = p.kb;
  plan[3] = p.pairs;
  return kOk;
}

// An upper bound of what any launch of this shape needs on this device (a
// launch may plan fewer pairs or a smaller token tile than a host-only query).
extern "C" int kvb_gemm_sk_workspace_size(int M, int N, int K, int gated, size_t* bytes) {
  if (!bytes || M < 0 || N <= 0 || K <= 0) return set_error(kInvalid, "kvb_gemm_sk_workspace_size: bad sizes");
  (void)gated;
  const size_t pairs = (size_t)std::min(kMaxPairs, device_sm_count() / 2);
  *bytes = M == 0 ? 0 : kFlagBytes + pairs * 2 * kRows * token_tile(M) * sizeof(float);
  return kOk;
}

extern "C" int kvb_gemm_sk_set_plan(int mt, int pairs) {
  if ((mt != 0 && mt != 16 && mt != 32 && mt != 64 && mt != 128 && mt != 256) || pairs < 0 || pairs > kMaxPairs)
    return set_error(kInvalid, "kvb_gemm_sk_set_plan: token tile 0/16/32/64/128/256, pairs 0..%d", kMaxPairs);
  g_sk_force_mt.store(mt);
  g_sk_force_pairs.store(pairs);
  return kOk;
}

extern "C" int kvb_gemm_sk_bf16(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy, int M,
                                int N, int K, void* workspace, size_t workspace_bytes, void* stream) {
  return run_sk(x, ldx, w, ldw, y, ldy, M, N, K, workspace, workspace_bytes, stream, false, "kvb_gemm_sk_bf16");
}

extern "C" int kvb_gemm_sk_silu_bf16(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy,
                                     int M, int inter, int K, void* workspace, size_t workspace_bytes, void* stream) {
  return run_sk(x, ldx, w, ldw, y, ldy, M, inter, K, workspace, workspace_bytes, stream, true,
                "kvb_gemm_sk_silu_bf16");
}
