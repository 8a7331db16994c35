// Causal varlen prefill attention (flash_attention_kvcache.py:73-79:
// flash_attn_varlen_func(q, k, v, cu_seqlens_q/k, max_seqlen_q/k, causal=True,
// block_table)). Bottom-right causal alignment: query i of a sequence with
// seqlen_q new tokens over kv_len keys sits at position kv_len - seqlen_q + i
// and sees keys [0, kv_len - seqlen_q + i].
//
// Two kernels:
// * prefill_tc_kernel (the default): 5th-generation tensor cores. A CTA owns
//   128 query rows of one head; per 128-key tile S = Q K^T is one
//   tcgen05.mma (M=128, N=128, K=128 in 8 steps) into TMEM (two S buffers,
//   so the next tile's QK^T overlaps this tile's softmax), the four softmax
//   warps own one query row per thread (TMEM lane = row: no cross-thread
//   reductions), write P (bf16) to shared memory, and O_tile = P V is a second
//   tcgen05.mma (V read MN-major straight from its TMA tile) into a third TMEM
//   buffer that each thread folds into its fp32 O row (online softmax, exp2
//   domain). Q/K/V arrive by TMA (3-D maps over the token rows, or 4-D maps
//   over the paged cache with the block id from the block table), 128-byte
//   swizzle, a 2-stage K/V ring. Used when the page size is a multiple of 128.
// * prefill_attn_kernel (other page sizes), the warp-MMA generation:
//   grid  = (query tiles of 64 rows, Hq, batch), heaviest causal tiles first;
//   CTA   = 4 warps, each owns 16 query rows of one head;
//   K/V   = 64-key tiles double-buffered in 128-byte-swizzled shared memory by
//           cp.async, read either through the block table from the paged cache
//           (prefix cache / chunked prefill) or from contiguous k/v rows;
//   math  = bf16 m16n8k16 MMAs, fp32 online softmax (exp2 domain), P rounded
//           to bf16 for the PV product as FlashAttention-2 does.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "../../include/kavor_b200.h"

KVB_DEFINE_ERROR_WORD(prefill)

namespace kvb {
namespace {

constexpr int kHD = 128;
constexpr int kRows = 64;   // query rows per CTA
constexpr int kKeys = 64;   // keys per tile
constexpr int kThreads = 128;
constexpr int kRowBytes = kHD * 2;               // 256
constexpr int kTileBytes = kKeys * kRowBytes;    // 16 KB
constexpr int kSmemBytes = kRows * kRowBytes + 4 * kTileBytes + 128;  // Q + 2x(K,V)

struct PrefillArgs {
  const bf16* q;
  int64_t q_st, q_sh;
  const bf16* k;
  int64_t k_st, k_sh;
  const bf16* v;
  int64_t v_st, v_sh;
  int64_t num_blocks, block_stride;
  int block_size;
  const int32_t* block_tables;
  int64_t bt_stride;
  int max_blocks;
  const int32_t* cu_q;
  const int32_t* cu_k;
  bf16* out;
  int64_t o_st, o_sh;
  int hkv, group;
  float scale_log2;
};

// 16-byte chunk c (0..15) of row r of a [rows][256 B] tile
__device__ __forceinline__ uint32_t swz(uint32_t base, int row, int chunk) {
  return base + row * kRowBytes + ((chunk ^ (row & 7)) << 4);
}

template <bool kPaged>
__device__ __forceinline__ void load_kv_tile(const PrefillArgs& a, int b, int kvh, int key0, int kv_len, int k_off,
                                             uint32_t kdst, uint32_t vdst) {
  const int chunk = threadIdx.x & 15;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int row = (threadIdx.x >> 4) + i * 8;
    const int key = key0 + row;
    bool valid = key < kv_len;
    const bf16* ks = a.k;
    const bf16* vs = a.v;
    if (valid) {
      if constexpr (kPaged) {
        const int col = key / a.block_size;
        const int blk = col < a.max_blocks ? a.block_tables[(int64_t)b * a.bt_stride + col] : -1;
        if (blk < 0 || blk >= a.num_blocks) {
          atomicOr(&g_err_prefill, (unsigned)kErrBlockTable);
          valid = false;
        } else {
          const int64_t off = (int64_t)blk * a.block_stride +
                              ((int64_t)(key - col * a.block_size) * a.hkv + kvh) * kHD + chunk * 8;
          ks = a.k + off;
          vs = a.v + off;
        }
      } else {
        const int64_t t = (int64_t)k_off + key;
        ks = a.k + t * a.k_st + (int64_t)kvh * a.k_sh + chunk * 8;
        vs = a.v + t * a.v_st + (int64_t)kvh * a.v_sh + chunk * 8;
      }
    }
    cp_async_16(swz(kdst, row, chunk), ks, valid);
    cp_async_16(swz(vdst, row, chunk), vs, valid);
  }
}

template <bool kPaged>
__global__ void __launch_bounds__(kThreads, 2) prefill_attn_kernel(const __grid_constant__ PrefillArgs a) {
  kernel_entry();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const int qtile = gridDim.x - 1 - blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int q_seq0 = a.cu_q[b];
  const int seqlen_q = a.cu_q[b + 1] - q_seq0;
  const int q0 = qtile * kRows;
  if (q0 >= seqlen_q) return;
  const int k_off = a.cu_k[b];
  const int kv_len = a.cu_k[b + 1] - k_off;
  const int delta = kv_len - seqlen_q;
  const int kvh = h / a.group;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  int kend = delta + min(q0 + kRows, seqlen_q);  // exclusive bound of visible keys for this tile
  if (kend > kv_len) kend = kv_len;
  const int ntiles = kend > 0 ? (kend + kKeys - 1) / kKeys : 0;

  const uint32_t qs = smem_u32(smem);
  const uint32_t kbuf[2] = {qs + kRows * kRowBytes, qs + kRows * kRowBytes + 2 * kTileBytes};
  const uint32_t vbuf[2] = {kbuf[0] + kTileBytes, kbuf[1] + kTileBytes};

  {  // Q tile
    const int chunk = threadIdx.x & 15;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int row = (threadIdx.x >> 4) + i * 8;
      const bool valid = q0 + row < seqlen_q;
      const bf16* src = a.q + (int64_t)(q_seq0 + (valid ? q0 + row : 0)) * a.q_st + (int64_t)h * a.q_sh + chunk * 8;
      cp_async_16(swz(qs, row, chunk), src, valid);
    }
  }
  if (ntiles > 0) load_kv_tile<kPaged>(a, b, kvh, 0, kv_len, k_off, kbuf[0], vbuf[0]);
  cp_async_commit();

  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  uint32_t qa[8][4];
  const int qi0 = q0 + warp * 16 + (lane >> 2);  // query rows of c0/c1 and c2/c3: qi0, qi0 + 8
  const int lim0 = delta + qi0, lim1 = delta + qi0 + 8;

  for (int j = 0; j < ntiles; ++j) {
    if (j + 1 < ntiles) {
      load_kv_tile<kPaged>(a, b, kvh, (j + 1) * kKeys, kv_len, k_off, kbuf[(j + 1) & 1], vbuf[(j + 1) & 1]);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (j == 0) {
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const int m = lane >> 3;
        const int row = warp * 16 + (lane & 7) + ((m & 1) << 3);
        ldmatrix_x4(swz(qs, row, ks * 2 + (m >> 1)), qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3]);
      }
    }
    const uint32_t kb = kbuf[j & 1], vb = vbuf[j & 1];
    float sc[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        const int m = lane >> 3;
        const int row = np * 16 + (lane & 7) + ((m >> 1) << 3);
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(swz(kb, row, ks * 2 + (m & 1)), b0, b1, b2, b3);
        mma_bf16_16816(sc[2 * np], qa[ks], b0, b1);
        mma_bf16_16816(sc[2 * np + 1], qa[ks], b2, b3);
      }
    }
    const int key0 = j * kKeys;
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = key0 + n * 8 + (lane & 3) * 2 + e;
        const bool in = key < kv_len;
        sc[n][e] = (in && key <= lim0) ? sc[n][e] * a.scale_log2 : -INFINITY;
        sc[n][2 + e] = (in && key <= lim1) ? sc[n][2 + e] * a.scale_log2 : -INFINITY;
        mx0 = fmaxf(mx0, sc[n][e]);
        mx1 = fmaxf(mx1, sc[n][2 + e]);
      }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m_run[0], mx0), mn1 = fmaxf(m_run[1], mx1);
    const float b0s = mn0 == -INFINITY ? 0.f : mn0, b1s = mn1 == -INFINITY ? 0.f : mn1;
    const float c0 = exp2f(m_run[0] - b0s), c1 = exp2f(m_run[1] - b1s);
    m_run[0] = mn0;
    m_run[1] = mn1;
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      sc[n][0] = exp2f(sc[n][0] - b0s);
      sc[n][1] = exp2f(sc[n][1] - b0s);
      sc[n][2] = exp2f(sc[n][2] - b1s);
      sc[n][3] = exp2f(sc[n][3] - b1s);
      s0 += sc[n][0] + sc[n][1];
      s1 += sc[n][2] + sc[n][3];
    }
    l_run[0] = l_run[0] * c0 + s0;
    l_run[1] = l_run[1] * c1 + s1;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      o[n][0] *= c0;
      o[n][1] *= c0;
      o[n][2] *= c1;
      o[n][3] *= c1;
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t pa[4] = {pack_bf16(sc[2 * kk][0], sc[2 * kk][1]), pack_bf16(sc[2 * kk][2], sc[2 * kk][3]),
                              pack_bf16(sc[2 * kk + 1][0], sc[2 * kk + 1][1]),
                              pack_bf16(sc[2 * kk + 1][2], sc[2 * kk + 1][3])};
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        const int m = lane >> 3;
        const int row = kk * 16 + (lane & 7) + ((m & 1) << 3);
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(swz(vb, row, dp * 2 + (m >> 1)), b0, b1, b2, b3);
        mma_bf16_16816(o[2 * dp], pa, b0, b1);
        mma_bf16_16816(o[2 * dp + 1], pa, b2, b3);
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();  // no copy may outlive the CTA (ntiles == 0 leaves the Q group pending)

  l_run[0] += __shfl_xor_sync(0xffffffffu, l_run[0], 1);
  l_run[0] += __shfl_xor_sync(0xffffffffu, l_run[0], 2);
  l_run[1] += __shfl_xor_sync(0xffffffffu, l_run[1], 1);
  l_run[1] += __shfl_xor_sync(0xffffffffu, l_run[1], 2);
  const float inv0 = l_run[0] > 0.f ? 1.f / l_run[0] : 0.f;
  const float inv1 = l_run[1] > 0.f ? 1.f / l_run[1] : 0.f;
  const int d0 = (lane & 3) * 2;
  if (qi0 < seqlen_q) {
    bf16* orow = a.out + (int64_t)(q_seq0 + qi0) * a.o_st + (int64_t)h * a.o_sh + d0;
#pragma unroll
    for (int n = 0; n < 16; ++n)
      *reinterpret_cast<__nv_bfloat162*>(orow + n * 8) = __floats2bfloat162_rn(o[n][0] * inv0, o[n][1] * inv0);
  }
  if (qi0 + 8 < seqlen_q) {
    bf16* orow = a.out + (int64_t)(q_seq0 + qi0 + 8) * a.o_st + (int64_t)h * a.o_sh + d0;
#pragma unroll
    for (int n = 0; n < 16; ++n)
      *reinterpret_cast<__nv_bfloat162*>(orow + n * 8) = __floats2bfloat162_rn(o[n][2] * inv1, o[n][3] * inv1);
  }
}


// =====================================================================
// tcgen05 prefill kernel
// =====================================================================
constexpr int kTcThreads = 192;                 // warp 0 TMA, warp 1 MMA + TMEM, warps 2..5 softmax
constexpr int kTcRows = 128;                    // query rows per CTA (UMMA M)
constexpr int kTcKeys = 128;                    // keys per tile (UMMA N of QK^T, K of PV)
constexpr int kTcHalf = 128 * 64 * 2;           // [128 rows][64 bf16] 128-byte-swizzled half tile
constexpr int kTcTile = 2 * kTcHalf;            // 32 KB: 128 rows x 128 bf16
constexpr int kTcQ = 0, kTcK = kTcTile, kTcV = 3 * kTcTile, kTcP = 5 * kTcTile;  // K, V, P: 2 buffers each
constexpr int kTcSmem = 7 * kTcTile + 1024;     // 225 KB
constexpr uint32_t kTcCols = 512;               // TMEM: S0, S1, PV0, PV1 (128 columns each)

struct TcArgs {
  int block_size;
  const int32_t* block_tables;
  int64_t bt_stride;
  int max_blocks;
  int64_t num_blocks;
  const int32_t* cu_q;
  const int32_t* cu_k;
  bf16* out;
  int64_t o_st, o_sh;
  int group;
  float scale_log2;
  uint32_t idesc_qk, idesc_pv;
};

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tma_load_4d_plain(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                                  uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
      : "memory");
}

// K-major operand, 128-byte swizzle: 8-row groups 1024 B apart (SBO), LBO
// unused; sm100 descriptor version 1, layout type 2.
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// MN-major operand (V as the B operand of P V: head_dim contiguous), 128-byte
// swizzle: 64-element atoms along head_dim kTcHalf bytes apart (LBO, the two
// TMA halves), 8-key groups 1024 B apart (SBO).
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)(kTcHalf >> 4) << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
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

template <bool kPaged>
__global__ void __launch_bounds__(kTcThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap, const __grid_constant__ TcArgs a) {
  kernel_entry();
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t q_full, kfull[2], vfull[2], kv_empty[2], s_full[2], s_empty[2], p_full[2],
      pv_full[2], pv_empty[2];
  __shared__ uint32_t tmem_s;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const int qtile = gridDim.x - 1 - blockIdx.x;  // heaviest causal tiles first
  const int h = blockIdx.y, b = blockIdx.z;
  const int q_seq0 = a.cu_q[b];
  const int seqlen_q = a.cu_q[b + 1] - q_seq0;
  const int q0 = qtile * kTcRows;
  if (q0 >= seqlen_q) return;  // uniform for the CTA, before any barrier or TMEM use
  const int k_off = a.cu_k[b];
  const int kv_len = a.cu_k[b + 1] - k_off;
  const int delta = kv_len - seqlen_q;  // bottom-right causal alignment
  const int kvh = h / a.group;
  int kend = delta + min(q0 + kTcRows, seqlen_q);
  if (kend > kv_len) kend = kv_len;
  const int ntiles = kend > 0 ? (kend + kTcKeys - 1) / kTcKeys : 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&q_full), 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&kfull[i]), 1);
      mbar_init(smem_u32(&vfull[i]), 1);
      mbar_init(smem_u32(&kv_empty[i]), 1);
      mbar_init(smem_u32(&s_full[i]), 1);
      mbar_init(smem_u32(&s_empty[i]), 4);
      mbar_init(smem_u32(&p_full[i]), 4);
      mbar_init(smem_u32(&pv_full[i]), 1);
      mbar_init(smem_u32(&pv_empty[i]), 4);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_s)),
                 "r"(kTcCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_before();
  __syncthreads();
  tc_after();
  const uint32_t tmem = tmem_s;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0 && ntiles > 0) {
      prefetch_tensormap(&qmap);
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
      mbar_arrive_expect_tx(smem_u32(&q_full), kTcTile);
      for (int hf = 0; hf < 2; ++hf)
        tma_load_3d(sbase + kTcQ + hf * kTcHalf, &qmap, hf * 64, h, q_seq0 + q0, smem_u32(&q_full));
      int issued = 0;
      for (int j = 0; j < ntiles; ++j) {
        const int st = j & 1;
        if (j >= 2 && !mbar_wait(smem_u32(&kv_empty[st]), ((j >> 1) - 1) & 1, &g_err_prefill)) break;
        const int key0 = j * kTcKeys;
        int c2, c3 = 0;
        if constexpr (kPaged) {
          const int col = key0 / a.block_size;
          int blk = col < a.max_blocks ? a.block_tables[(int64_t)b * a.bt_stride + col] : -1;
          if (blk < 0 || blk >= a.num_blocks) {
            atomicOr(&g_err_prefill, (unsigned)kErrBlockTable);
            blk = (int)a.num_blocks;  // out of range: the TMA reads zeros
          }
          c2 = key0 - col * a.block_size;
          c3 = blk;
        } else {
          c2 = k_off + key0;
        }
        const uint32_t kb = smem_u32(&kfull[st]), vb = smem_u32(&vfull[st]);
        mbar_arrive_expect_tx(kb, kTcTile);
        for (int hf = 0; hf < 2; ++hf) {
          if constexpr (kPaged) tma_load_4d_plain(sbase + kTcK + st * kTcTile + hf * kTcHalf, &kmap, hf * 64, kvh, c2, c3, kb);
          else tma_load_3d(sbase + kTcK + st * kTcTile + hf * kTcHalf, &kmap, hf * 64, kvh, c2, kb);
        }
        mbar_arrive_expect_tx(vb, kTcTile);
        for (int hf = 0; hf < 2; ++hf) {
          if constexpr (kPaged) tma_load_4d_plain(sbase + kTcV + st * kTcTile + hf * kTcHalf, &vmap, hf * 64, kvh, c2, c3, vb);
          else tma_load_3d(sbase + kTcV + st * kTcTile + hf * kTcHalf, &vmap, hf * 64, kvh, c2, vb);
        }
        issued = j + 1;
      }
      // no copy may outlive the CTA: wait (bounded) for the last stages' bytes,
      // which the MMA warp has normally consumed already
      for (int j = issued - 2 < 0 ? 0 : issued - 2; j < issued; ++j) {
        mbar_wait(smem_u32(&kfull[j & 1]), (j >> 1) & 1, &g_err_prefill);
        mbar_wait(smem_u32(&vfull[j & 1]), (j >> 1) & 1, &g_err_prefill);
      }
      mbar_wait(smem_u32(&q_full), 0, &g_err_prefill);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && ntiles > 0) {
      bool ok = mbar_wait(smem_u32(&q_full), 0, &g_err_prefill);
      auto issue_s = [&](int j) -> bool {
        const int sb = j & 1, st = j & 1;
        if (j >= 2 && !mbar_wait(smem_u32(&s_empty[sb]), ((j >> 1) - 1) & 1, &g_err_prefill)) return false;
        if (!mbar_wait(smem_u32(&kfull[st]), (j >> 1) & 1, &g_err_prefill)) return false;
        tc_after();
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint32_t off = (ks >> 2) * kTcHalf + (ks & 3) * 32;  // K = head_dim: 16 per step
          tc_mma(tmem + sb * kTcKeys, desc_kmajor(sbase + kTcQ + off), desc_kmajor(sbase + kTcK + st * kTcTile + off),
                 a.idesc_qk, ks > 0);
        }
        tc_commit(smem_u32(&s_full[sb]));
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; j < ntiles && ok; ++j) {
        if (j + 1 < ntiles && !issue_s(j + 1)) break;
        const int st = j & 1, pb = j & 1;  // K/V stage, P and PV buffers of tile j
        if (!mbar_wait(smem_u32(&p_full[pb]), (j >> 1) & 1, &g_err_prefill)) break;
        if (!mbar_wait(smem_u32(&vfull[st]), (j >> 1) & 1, &g_err_prefill)) break;
        if (j >= 2 && !mbar_wait(smem_u32(&pv_empty[pb]), ((j >> 1) - 1) & 1, &g_err_prefill)) break;
        tc_after();
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {  // K = keys: 16 per step
          const uint32_t pa = sbase + kTcP + pb * kTcTile + (ks >> 2) * kTcHalf + (ks & 3) * 32;
          const uint32_t vb = sbase + kTcV + st * kTcTile + ks * 2048;
          tc_mma(tmem + (2 + pb) * kTcKeys, desc_kmajor(pa), desc_mnmajor(vb), a.idesc_pv, ks > 0);
        }
        tc_commit(smem_u32(&pv_full[pb]));
        tc_commit(smem_u32(&kv_empty[st]));
      }
    }
  } else {
    // ------------------------------------------------------------ softmax warps
    const int qd = warp & 3;                 // TMEM lane quarter of this warp
    const int r = qd * 32 + lane;             // query row within the tile = TMEM lane
    const int qi = q0 + r;
    const int lim = delta + qi;               // last visible key of this row
    const uint32_t lane_base = tmem + ((uint32_t)(qd * 32) << 16);
    float o[kHD];
#pragma unroll
    for (int i = 0; i < kHD; ++i) o[i] = 0.f;
    float m_run = -INFINITY, l_run = 0.f;
    float corr_prev = 1.f;  // rescale of the tile whose P V is folded next
    bool ok = true;
    // fold P V of tile t (computed relative to that tile's max) into O
    auto fold = [&](int t, float corr) -> bool {
      const int pb = t & 1;
      if (!mbar_wait(smem_u32(&pv_full[pb]), (t >> 1) & 1, &g_err_prefill)) return false;
      tc_after();
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float v[32];
        tmem_ld32(lane_base + (2 + pb) * kTcKeys + c * 32, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) o[c * 32 + i] = o[c * 32 + i] * corr + v[i];
      }
      tc_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&pv_empty[pb]));
      return true;
    };
    for (int j = 0; j < ntiles && ok; ++j) {
      const int sb = j & 1, st = j & 1, pb = j & 1;
      const int key0 = j * kTcKeys;
      if (!mbar_wait(smem_u32(&s_full[sb]), (j >> 1) & 1, &g_err_prefill)) { ok = false; break; }
      tc_after();
      const uint32_t srow = lane_base + sb * kTcKeys;
      float mx = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float v[32];
        tmem_ld32(srow + c * 32, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int key = key0 + c * 32 + i;
          const float x = (key < kv_len && key <= lim) ? v[i] * a.scale_log2 : -INFINITY;
          mx = fmaxf(mx, x);
        }
      }
      const float m_new = fmaxf(m_run, mx);
      const float base = m_new == -INFINITY ? 0.f : m_new;
      const float corr = exp2f(m_run - base);
      float psum = 0.f;
      // P buffer pb was last read by P V of tile j - 2, folded (waited for)
      // in the previous iteration
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float v[32];
        tmem_ld32(srow + c * 32, v);
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const int key = key0 + c * 32 + i;
          const float x0 = (key < kv_len && key <= lim) ? v[i] * a.scale_log2 : -INFINITY;
          const float x1 = (key + 1 < kv_len && key + 1 <= lim) ? v[i + 1] * a.scale_log2 : -INFINITY;
          const float p0 = exp2f(x0 - base), p1 = exp2f(x1 - base);
          psum += p0 + p1;
          pk[i / 2] = pack_bf16(p0, p1);
        }
        // keys c*32 .. c*32+31 of row r: half c/2, 16-byte chunks (c%2)*4 .. +3
        const uint32_t prow = sbase + kTcP + pb * kTcTile + (c >> 1) * kTcHalf + r * 128;
#pragma unroll
        for (int k4 = 0; k4 < 4; ++k4) {
          const int ch = (c & 1) * 4 + k4;
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(prow + ((ch ^ (r & 7)) << 4)),
                       "r"(pk[4 * k4]), "r"(pk[4 * k4 + 1]), "r"(pk[4 * k4 + 2]), "r"(pk[4 * k4 + 3])
                       : "memory");
        }
      }
      tc_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&s_empty[sb]));
      if (key0 + kTcKeys > kv_len) {
        // keys past the sequence in the last tile: zero their V rows (stale
        // cache bytes may be NaN and P = 0 does not cancel NaN)
        if (!mbar_wait(smem_u32(&vfull[st]), (j >> 1) & 1, &g_err_prefill)) { ok = false; break; }
        if (key0 + r >= kv_len) {
#pragma unroll
          for (int hf = 0; hf < 2; ++hf)
#pragma unroll
            for (int ch = 0; ch < 8; ++ch)
              asm volatile("st.shared.v4.b32 [%0], {%1, %1, %1, %1};" ::"r"(sbase + kTcV + st * kTcTile + hf * kTcHalf +
                                                                           r * 128 + ch * 16),
                           "r"(0u)
                           : "memory");
        }
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&p_full[pb]));
      l_run = l_run * corr + psum;
      m_run = m_new;
      // P V of this tile now runs on the tensor core; fold the previous one
      if (j >= 1 && !fold(j - 1, corr_prev)) { ok = false; break; }
      corr_prev = corr;
    }
    if (ok && ntiles > 0 && !fold(ntiles - 1, corr_prev)) ok = false;
    if (qi < seqlen_q) {
      const float inv = (ok && l_run > 0.f) ? 1.f / l_run : 0.f;
      bf16* orow = a.out + (int64_t)(q_seq0 + qi) * a.o_st + (int64_t)h * a.o_sh;
#pragma unroll
      for (int c = 0; c < kHD / 8; ++c) {
        uint4 pk;
        pk.x = pack_bf16(o[8 * c] * inv, o[8 * c + 1] * inv);
        pk.y = pack_bf16(o[8 * c + 2] * inv, o[8 * c + 3] * inv);
        pk.z = pack_bf16(o[8 * c + 4] * inv, o[8 * c + 5] * inv);
        pk.w = pack_bf16(o[8 * c + 6] * inv, o[8 * c + 7] * inv);
        *reinterpret_cast<uint4*>(orow + 8 * c) = pk;
      }
    }
  }
  tc_before();
  __syncthreads();
  if (warp == 1) {
    tc_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcCols) : "memory");
  }
}

// rows of `heads` x 128 bf16 (head stride `sh`, row stride `st`, elements): box
// {64 dims, 1 head, 128 rows}; 4-D form for the paged cache: {128, heads,
// block_size, num_blocks} with block stride `bst`.
int encode_rows(CUtensorMap* map, const void* base, int heads, int64_t rows, int64_t sh, int64_t st) {
  auto enc = tensor_map_encoder();
  if (!enc) return set_error(kNoEncoder, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[3] = {(cuuint64_t)kHD, (cuuint64_t)heads, (cuuint64_t)rows};
  const cuuint64_t strides[2] = {(cuuint64_t)sh * 2, (cuuint64_t)st * 2};
  const cuuint32_t box[3] = {64, 1, (cuuint32_t)kTcRows};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(kEncode, "cuTensorMapEncodeTiled (3-D) failed (CUresult %d)", (int)r);
  return kOk;
}

int encode_pages(CUtensorMap* map, const void* base, int hkv, int block_size, int64_t num_blocks, int64_t bst) {
  auto enc = tensor_map_encoder();
  if (!enc) return set_error(kNoEncoder, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[4] = {(cuuint64_t)kHD, (cuuint64_t)hkv, (cuuint64_t)block_size, (cuuint64_t)num_blocks};
  const cuuint64_t strides[3] = {(cuuint64_t)kHD * 2, (cuuint64_t)hkv * kHD * 2, (cuuint64_t)bst * 2};
  const cuuint32_t box[4] = {64, 1, (cuuint32_t)kTcKeys, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(kEncode, "cuTensorMapEncodeTiled (4-D) failed (CUresult %d)", (int)r);
  return kOk;
}

template <bool kPaged>
int launch_tc(const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm, const TcArgs& a, dim3 grid,
              cudaStream_t st) {
  static unsigned long long done = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !((done >> dev) & 1ull)) {
    cudaError_t e = cudaFuncSetAttribute(prefill_tc_kernel<kPaged>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
    if (e != cudaSuccess) return cuda_status(e, "prefill tc smem attribute");
    if (dev < 64) done |= 1ull << dev;
  }
  return cuda_status(launch_kernel(prefill_tc_kernel<kPaged>, grid, dim3(kTcThreads), kTcSmem, st, qm, km, vm, a),
                     "kvb_prefill_attn (tcgen05) launch");
}

template <bool kPaged>
int ensure_attr() {
  static unsigned long long done = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
  if (dev < 64 && (done >> dev) & 1ull) return kOk;
  e = cudaFuncSetAttribute(prefill_attn_kernel<kPaged>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (e != cudaSuccess) return cuda_status(e, "prefill attention smem attribute");
  if (dev < 64) done |= 1ull << dev;
  return kOk;
}

}  // namespace
}  // namespace kvb

using namespace kvb;

extern "C" int kvb_prefill_attn(const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* k,
                                int64_t k_stride_t, int64_t k_stride_h, const void* v, int64_t v_stride_t,
                                int64_t v_stride_h, int64_t num_blocks, int64_t block_stride, int block_size,
                                const int32_t* block_tables, int64_t block_table_stride, int max_blocks_per_seq,
                                const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k, int batch, int max_seqlen_q,
                                void* out, int64_t out_stride_t, int64_t out_stride_h, int num_q_heads,
                                int num_kv_heads, int head_dim, float scale, int64_t total_q, int64_t total_k,
                                void* stream) {
  if (batch < 0 || max_seqlen_q < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads)
    return set_error(kInvalid, "kvb_prefill_attn: bad sizes");
  if (head_dim != kHD) return set_error(kUnsupported, "kvb_prefill_attn: head_dim must be 128");
  if (batch == 0 || max_seqlen_q == 0) return kOk;
  if (!q || !k || !v || !cu_seqlens_q || !cu_seqlens_k || !out)
    return set_error(kInvalid, "kvb_prefill_attn: NULL pointer");
  if (((uintptr_t)q & 15) || q_stride_t % 8 || q_stride_h % 8 || ((uintptr_t)out & 3) || out_stride_t % 2 ||
      out_stride_h % 2)
    return set_error(kInvalid, "kvb_prefill_attn: q rows must be 16-byte aligned");
  if (((uintptr_t)k & 15) || ((uintptr_t)v & 15)) return set_error(kInvalid, "kvb_prefill_attn: k/v alignment");
  const bool paged = block_tables != nullptr;
  if (paged) {
    if (block_size <= 0 || num_blocks <= 0 || max_blocks_per_seq <= 0 || block_stride % 8 ||
        block_stride < (int64_t)block_size * num_kv_heads * kHD)
      return set_error(kInvalid, "kvb_prefill_attn: bad paged-cache arguments");
  } else if (k_stride_t % 8 || k_stride_h % 8 || v_stride_t % 8 || v_stride_h % 8) {
    return set_error(kInvalid, "kvb_prefill_attn: k/v rows must be 16-byte aligned");
  }
  PrefillArgs a;
  a.q = (const bf16*)q;
  a.q_st = q_stride_t;
  a.q_sh = q_stride_h;
  a.k = (const bf16*)k;
  a.k_st = k_stride_t;
  a.k_sh = k_stride_h;
  a.v = (const bf16*)v;
  a.v_st = v_stride_t;
  a.v_sh = v_stride_h;
  a.num_blocks = num_blocks;
  a.block_stride = block_stride;
  a.block_size = block_size;
  a.block_tables = block_tables;
  a.bt_stride = block_table_stride;
  a.max_blocks = max_blocks_per_seq;
  a.cu_q = cu_seqlens_q;
  a.cu_k = cu_seqlens_k;
  a.out = (bf16*)out;
  a.o_st = out_stride_t;
  a.o_sh = out_stride_h;
  a.hkv = num_kv_heads;
  a.group = num_q_heads / num_kv_heads;
  a.scale_log2 = scale * 1.4426950408889634f;
  // tensor-core kernel: needs the row extents for its TMA maps, pages of a
  // multiple of 128 tokens, and 16-byte output rows
  const bool tc = total_q > 0 && (paged ? block_size % kTcKeys == 0 : total_k > 0) && ((uintptr_t)out & 15) == 0 &&
                  out_stride_t % 8 == 0 && out_stride_h % 8 == 0;
  if (tc) {
    CUtensorMap qm, km, vm;
    int rc = encode_rows(&qm, q, num_q_heads, total_q, q_stride_h, q_stride_t);
    if (!rc)
      rc = paged ? encode_pages(&km, k, num_kv_heads, block_size, num_blocks, block_stride)
                 : encode_rows(&km, k, num_kv_heads, total_k, k_stride_h, k_stride_t);
    if (!rc)
      rc = paged ? encode_pages(&vm, v, num_kv_heads, block_size, num_blocks, block_stride)
                 : encode_rows(&vm, v, num_kv_heads, total_k, v_stride_h, v_stride_t);
    if (rc) return rc;
    TcArgs t;
    t.block_size = block_size;
    t.block_tables = block_tables;
    t.bt_stride = block_table_stride;
    t.max_blocks = max_blocks_per_seq;
    t.num_blocks = num_blocks;
    t.cu_q = cu_seqlens_q;
    t.cu_k = cu_seqlens_k;
    t.out = (bf16*)out;
    t.o_st = out_stride_t;
    t.o_sh = out_stride_h;
    t.group = num_q_heads / num_kv_heads;
    t.scale_log2 = a.scale_log2;
    // kind::f16 instruction descriptors: fp32 D, bf16 A and B, M=128, N=128;
    // P V reads B (= V) MN-major (bit 16)
    const uint32_t base = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kTcKeys >> 3) << 17) | ((uint32_t)(kTcRows >> 4) << 24);
    t.idesc_qk = base;
    t.idesc_pv = base | (1u << 16);
    dim3 g((max_seqlen_q + kTcRows - 1) / kTcRows, num_q_heads, batch);
    return paged ? launch_tc<true>(qm, km, vm, t, g, (cudaStream_t)stream)
                 : launch_tc<false>(qm, km, vm, t, g, (cudaStream_t)stream);
  }
  dim3 grid((max_seqlen_q + kRows - 1) / kRows, num_q_heads, batch);
  int rc = paged ? ensure_attr<true>() : ensure_attr<false>();
  if (rc) return rc;
  const cudaError_t e =
      paged ? launch_kernel(prefill_attn_kernel<true>, grid, dim3(kThreads), kSmemBytes, (cudaStream_t)stream, a)
            : launch_kernel(prefill_attn_kernel<false>, grid, dim3(kThreads), kSmemBytes, (cudaStream_t)stream, a);
  return cuda_status(e, "kvb_prefill_attn launch");
}
