// Causal varlen prefill attention (flash_attention_kvcache.py:73-79:
// flash_attn_varlen_func(q, k, v, cu_seqlens_q/k, max_seqlen_q/k, causal=True,
// block_table)). Bottom-right causal alignment: query i of a sequence with
// seqlen_q new tokens over kv_len keys sits at position kv_len - seqlen_q + i
// and sees keys [0, kv_len - seqlen_q + i].
//
// This is the first (warp-MMA) generation of the prefill kernel:
//   grid  = (query tiles of 64 rows, Hq, batch), heaviest causal tiles first;
//   CTA   = 4 warps, each owns 16 query rows of one head;
//   K/V   = 64-key tiles double-buffered in 128-byte-swizzled shared memory by
//           cp.async, read either through the block table from the paged cache
//           (prefix cache / chunked prefill) or from contiguous k/v rows;
//   math  = bf16 m16n8k16 MMAs, fp32 online softmax (exp2 domain), P rounded
//           to bf16 for the PV product as FlashAttention-2 does.
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
                                int num_kv_heads, int head_dim, float scale, void* stream) {
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
  dim3 grid((max_seqlen_q + kRows - 1) / kRows, num_q_heads, batch);
  int rc = paged ? ensure_attr<true>() : ensure_attr<false>();
  if (rc) return rc;
  if (paged)
    prefill_attn_kernel<true><<<grid, kThreads, kSmemBytes, (cudaStream_t)stream>>>(a);
  else
    prefill_attn_kernel<false><<<grid, kThreads, kSmemBytes, (cudaStream_t)stream>>>(a);
  return cuda_status(cudaGetLastError(), "kvb_prefill_attn launch");
}
