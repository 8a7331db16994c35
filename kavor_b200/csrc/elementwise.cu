// Memory-bound per-token kernels of the Qwen3 layer: KV-cache write, RMSNorm,
// add+RMSNorm, RoPE, the fused q/k-norm + RoPE + KV write, SiLU*mul and the
// vocab-sharded embedding lookup. All of them move 16-byte vectors (8 bf16)
// per thread where the row is contiguous, keep fp32 inside and round to bf16
// at exactly the points the reference rounds (layernorm.py:37,139 double
// rounding; rotary_embedding.py:50-53 fp32 rotation).
#include "common.cuh"
#include "../../include/kavor_b200.h"

KVB_DEFINE_ERROR_WORD(elementwise)

namespace kvb {
namespace {

struct alignas(16) Vec8 {
  __nv_bfloat162 h[4];
};

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

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ------------------------------------------------------------------ store_kv
// One warp per token; the row of num_kv_heads*head_dim elements is copied in
// 16-byte chunks (flash_attention_kvcache.py:23-34).
__global__ void store_kv_kernel(const bf16* __restrict__ key, int64_t key_stride, const bf16* __restrict__ value,
                                int64_t value_stride, bf16* __restrict__ k_cache, bf16* __restrict__ v_cache,
                                int64_t num_slots, int64_t block_stride, int block_size, int row_elems,
                                const int32_t* __restrict__ slot_mapping, int num_tokens) {
  kernel_entry();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= num_tokens) return;
  const int64_t slot = slot_mapping[warp];
  if (slot == -1) return;
  if (slot < 0 || slot >= num_slots) {
    if (lane == 0) atomicOr(&g_err_elementwise, (unsigned)kErrSlot);
    return;
  }
  const int64_t blk = slot / block_size, off = slot - blk * block_size;
  const int64_t dst = blk * block_stride + off * row_elems;
  const Vec8* ks = reinterpret_cast<const Vec8*>(key + (int64_t)warp * key_stride);
  const Vec8* vs = reinterpret_cast<const Vec8*>(value + (int64_t)warp * value_stride);
  Vec8* kd = reinterpret_cast<Vec8*>(k_cache + dst);
  Vec8* vd = reinterpret_cast<Vec8*>(v_cache + dst);
  for (int c = lane; c < row_elems / 8; c += 32) {
    kd[c] = ks[c];
    vd[c] = vs[c];
  }
}

// ------------------------------------------------------------------ RMSNorm
// head_dim == 128 rows (q/k norm): one warp per (token, head), 4 values/lane.
__global__ void rmsnorm128_kernel(const bf16* __restrict__ x, int64_t xst, int64_t xsh, bf16* __restrict__ out,
                                  int64_t ost, int64_t osh, const bf16* __restrict__ w, int tokens, int heads,
                                  float eps) {
  kernel_entry();
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= tokens * heads) return;
  const int t = row / heads, h = row - t * heads;
  const bf16* xr = x + (int64_t)t * xst + (int64_t)h * xsh + lane * 4;
  uint2 raw = *reinterpret_cast<const uint2*>(xr);
  const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&raw);
  float v[4];
  float2 a = __bfloat1622float2(p[0]), b = __bfloat1622float2(p[1]);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
  float ss = warp_sum(v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3]);
  const float rstd = rsqrtf(ss / 128.f + eps);
  uint2 wraw = *reinterpret_cast<const uint2*>(w + lane * 4);
  const __nv_bfloat162* wp = reinterpret_cast<const __nv_bfloat162*>(&wraw);
  float2 wa = __bfloat1622float2(wp[0]), wb = __bfloat1622float2(wp[1]);
  float wv[4] = {wa.x, wa.y, wb.x, wb.y};
  __nv_bfloat162 o[2];
  o[0] = __floats2bfloat162_rn(bf16_round(v[0] * rstd) * wv[0], bf16_round(v[1] * rstd) * wv[1]);
  o[1] = __floats2bfloat162_rn(bf16_round(v[2] * rstd) * wv[2], bf16_round(v[3] * rstd) * wv[3]);
  *reinterpret_cast<uint2*>(out + (int64_t)t * ost + (int64_t)h * osh + lane * 4) = *reinterpret_cast<uint2*>(o);
}

template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) s += red[i];
  return s;
}

// Generic rows (hidden sizes): one CTA of 256 threads per (token, head) row,
// each thread keeps up to MAXC 8-element chunks in registers.
constexpr int kRowThreads = 256;
constexpr int kRowMaxChunks = 8;  // n_cols <= 256 * 8 * 8 = 16384

__global__ void __launch_bounds__(kRowThreads) rmsnorm_row_kernel(const bf16* __restrict__ x, int64_t xst,
                                                                  int64_t xsh, bf16* __restrict__ out, int64_t ost,
                                                                  int64_t osh, const bf16* __restrict__ w,
                                                                  int heads, int n_cols, float eps) {
  kernel_entry();
  __shared__ float red[kRowThreads / 32];
  const int t = blockIdx.x / heads, h = blockIdx.x - (blockIdx.x / heads) * heads;
  const Vec8* xr = reinterpret_cast<const Vec8*>(x + (int64_t)t * xst + (int64_t)h * xsh);
  Vec8* orow = reinterpret_cast<Vec8*>(out + (int64_t)t * ost + (int64_t)h * osh);
  const Vec8* wr = reinterpret_cast<const Vec8*>(w);
  const int nch = n_cols / 8;
  float v[kRowMaxChunks][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kRowMaxChunks; ++i) {
    const int c = threadIdx.x + i * kRowThreads;
    if (c < nch) {
      unpack8(xr[c], v[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
    }
  }
  const float rstd = rsqrtf(block_sum<kRowThreads>(ss, red) / (float)n_cols + eps);
#pragma unroll
  for (int i = 0; i < kRowMaxChunks; ++i) {
    const int c = threadIdx.x + i * kRowThreads;
    if (c < nch) {
      float wf[8], y[8];
      unpack8(wr[c], wf);
#pragma unroll
      for (int j = 0; j < 8; ++j) y[j] = bf16_round(v[i][j] * rstd) * wf[j];
      orow[c] = pack8(y);
    }
  }
}

__global__ void __launch_bounds__(kRowThreads) add_rmsnorm_kernel(const bf16* __restrict__ x, bf16* residual,
                                                                  bf16* out, const bf16* __restrict__ w, int n_cols,
                                                                  float eps) {
  kernel_entry();
  __shared__ float red[kRowThreads / 32];
  const int64_t row = blockIdx.x;
  const Vec8* xr = reinterpret_cast<const Vec8*>(x + row * n_cols);
  Vec8* rr = reinterpret_cast<Vec8*>(residual + row * n_cols);
  Vec8* orow = reinterpret_cast<Vec8*>(out + row * n_cols);
  const Vec8* wr = reinterpret_cast<const Vec8*>(w);
  const int nch = n_cols / 8;
  float v[kRowMaxChunks][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kRowMaxChunks; ++i) {
    const int c = threadIdx.x + i * kRowThreads;
    if (c < nch) {
      float a[8], b[8];
      unpack8(xr[c], a);
      unpack8(rr[c], b);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[i][j] = a[j] + b[j];
        ss += v[i][j] * v[i][j];
      }
    }
  }
  const float rstd = rsqrtf(block_sum<kRowThreads>(ss, red) / (float)n_cols + eps);
#pragma unroll
  for (int i = 0; i < kRowMaxChunks; ++i) {
    const int c = threadIdx.x + i * kRowThreads;
    if (c < nch) {
      float wf[8], y[8];
      unpack8(wr[c], wf);
      rr[c] = pack8(v[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) y[j] = bf16_round(v[i][j] * rstd) * wf[j];
      orow[c] = pack8(y);
    }
  }
}

// ------------------------------------------------------------------ RoPE
__device__ __forceinline__ const float* cos_sin_row(const float* cs, const int64_t* positions, int t,
                                                    int64_t max_position, int head_dim) {
  int64_t pos = positions[t];
  pos = pos < 0 ? 0 : (pos >= max_position ? max_position - 1 : pos);
  return cs + pos * head_dim;
}

// Generic head_dim: one warp per (token, head), lanes stride over the pairs.
__global__ void rope_kernel(bf16* q, int64_t qst, int64_t qsh, bf16* k, int64_t kst, int64_t ksh,
                            const int64_t* __restrict__ positions, const float* __restrict__ cs,
                            int64_t max_position, int tokens, int q_heads, int k_heads, int head_dim,
                            int interleaved) {
  kernel_entry();
  const int heads = q_heads + k_heads;
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= tokens * heads) return;
  const int t = row / heads, h = row - t * heads;
  bf16* base = h < q_heads ? q + (int64_t)t * qst + (int64_t)h * qsh : k + (int64_t)t * kst + (int64_t)(h - q_heads) * ksh;
  const float* c = cos_sin_row(cs, positions, t, max_position, head_dim);
  const int half = head_dim / 2;
  for (int i = lane; i < half; i += 32) {
    const int o1 = interleaved ? 2 * i : i;
    const int o2 = interleaved ? 2 * i + 1 : i + half;
    const float x1 = __bfloat162float(base[o1]), x2 = __bfloat162float(base[o2]);
    const float cv = c[i], sv = c[half + i];
    base[o1] = __float2bfloat16_rn(x1 * cv - x2 * sv);
    base[o2] = __float2bfloat16_rn(x2 * cv + x1 * sv);
  }
}

// ------------------------------------------------- fused qk-norm + RoPE + KV write
// head_dim == 128. Warp per (token, head) over Hq q-heads, Hkv k-heads and Hkv
// v-heads of the packed qkv row. Lane owns dims [4*lane, 4*lane+4); the RoPE
// partner of dim d (neox: d +- 64) lives in lane ^ 16.
__global__ void qknorm_rope_store_kernel(bf16* qkv, int64_t qkv_stride, int tokens, int hq, int hkv,
                                         const bf16* __restrict__ qw, const bf16* __restrict__ kw, float eps,
                                         int apply_norm, const int64_t* __restrict__ positions,
                                         const float* __restrict__ cs, int64_t max_position, int interleaved,
                                         bf16* k_cache, bf16* v_cache, int64_t num_slots, int64_t block_stride,
                                         int block_size, const int32_t* __restrict__ slot_mapping) {
  kernel_entry();
  const int heads = hq + 2 * hkv;
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= tokens * heads) return;
  const int t = row / heads, h = row - t * heads;
  bf16* base = qkv + (int64_t)t * qkv_stride + (int64_t)h * 128 + lane * 4;
  uint2 raw = *reinterpret_cast<const uint2*>(base);
  int kind = h < hq ? 0 : (h < hq + hkv ? 1 : 2);  // 0 q, 1 k, 2 v
  if (kind < 2) {
    const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&raw);
    float2 a = __bfloat1622float2(p[0]), b = __bfloat1622float2(p[1]);
    float v[4] = {a.x, a.y, b.x, b.y};
    if (apply_norm) {
      const float ss = warp_sum(v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3]);
      const float rstd = rsqrtf(ss / 128.f + eps);
      const bf16* w = (kind == 0 ? qw : kw) + lane * 4;
      uint2 wraw = *reinterpret_cast<const uint2*>(w);
      const __nv_bfloat162* wp = reinterpret_cast<const __nv_bfloat162*>(&wraw);
      float2 wa = __bfloat1622float2(wp[0]), wb = __bfloat1622float2(wp[1]);
      const float wv[4] = {wa.x, wa.y, wb.x, wb.y};
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = bf16_round(bf16_round(v[j] * rstd) * wv[j]);
    }
    const float* c = cos_sin_row(cs, positions, t, max_position, 128);
    float y[4];
    if (interleaved) {
      // pairs (d, d+1) and (d+2, d+3) are local; frequency index d/2
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int i = lane * 2 + j;
        const float cv = c[i], sv = c[64 + i];
        y[2 * j] = v[2 * j] * cv - v[2 * j + 1] * sv;
        y[2 * j + 1] = v[2 * j + 1] * cv + v[2 * j] * sv;
      }
    } else {
      const bool first = lane < 16;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float other = __shfl_xor_sync(0xffffffffu, v[j], 16);
        const int i = (lane & 15) * 4 + j;
        const float cv = c[i], sv = c[64 + i];
        y[j] = first ? v[j] * cv - other * sv : v[j] * cv + other * sv;
      }
    }
    __nv_bfloat162 o[2] = {__floats2bfloat162_rn(y[0], y[1]), __floats2bfloat162_rn(y[2], y[3])};
    raw = *reinterpret_cast<uint2*>(o);
    *reinterpret_cast<uint2*>(base) = raw;
  }
  if (kind > 0 && k_cache != nullptr) {
    const int64_t slot = slot_mapping[t];
    if (slot == -1) return;
    if (slot < 0 || slot >= num_slots) {
      if (lane == 0) atomicOr(&g_err_elementwise, (unsigned)kErrSlot);
      return;
    }
    const int64_t blk = slot / block_size, off = slot - blk * block_size;
    const int kvh = h - hq - (kind == 2 ? hkv : 0);
    bf16* dst = (kind == 1 ? k_cache : v_cache) + blk * block_stride + (off * hkv + kvh) * 128 + lane * 4;
    *reinterpret_cast<uint2*>(dst) = raw;
  }
}

// ------------------------------------------------------------------ SiLU*mul
__global__ void silu_mul_kernel(const bf16* __restrict__ x, int64_t xst, bf16* __restrict__ out, int64_t ost,
                                int tokens, int inter) {
  kernel_entry();
  const int nch = inter / 8;
  const int64_t total = (int64_t)tokens * nch;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / nch;
    const int c = (int)(i - t * nch);
    const Vec8* row = reinterpret_cast<const Vec8*>(x + t * xst);
    float g[8], u[8], y[8];
    unpack8(row[c], g);
    unpack8(row[c + nch], u);
#pragma unroll
    for (int j = 0; j < 8; ++j) y[j] = g[j] / (1.f + __expf(-g[j])) * u[j];
    reinterpret_cast<Vec8*>(out + t * ost)[c] = pack8(y);
  }
}

// ------------------------------------------------------------------ embedding
__global__ void embedding_kernel(const int64_t* __restrict__ ids, const bf16* __restrict__ w, bf16* __restrict__ out,
                                 int hidden, int64_t vocab_start, int64_t vocab_end, int64_t vocab_size) {
  kernel_entry();
  const int t = blockIdx.x;
  const int64_t id = ids[t];
  if (vocab_size > 0 && (id < 0 || id >= vocab_size) && threadIdx.x == 0)
    atomicOr(&g_err_elementwise, (unsigned)kErrTokenId);
  const bool hit = id >= vocab_start && id < vocab_end;
  const Vec8* src = reinterpret_cast<const Vec8*>(w + (hit ? (id - vocab_start) : 0) * (int64_t)hidden);
  Vec8* dst = reinterpret_cast<Vec8*>(out + (int64_t)t * hidden);
  Vec8 zero;
  const float zf[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  zero = pack8(zf);
  for (int c = threadIdx.x; c < hidden / 8; c += blockDim.x) dst[c] = hit ? src[c] : zero;
}

inline unsigned blocks_for(int64_t warps, int warps_per_block) {
  return (unsigned)((warps + warps_per_block - 1) / warps_per_block);
}

}  // namespace
}  // namespace kvb

using namespace kvb;

extern "C" int kvb_store_kv(const void* key, int64_t key_stride, const void* value, int64_t value_stride,
                            void* k_cache, void* v_cache, int64_t num_blocks, int64_t block_stride, int block_size,
                            int num_kv_heads, int head_dim, const int32_t* slot_mapping, int num_tokens,
                            void* stream) {
  if (num_tokens < 0 || num_kv_heads <= 0 || head_dim <= 0 || block_size <= 0 || num_blocks < 0)
    return set_error(kInvalid, "kvb_store_kv: bad sizes");
  if (num_tokens == 0) return kOk;
  const int row = num_kv_heads * head_dim;
  if (!key || !value || !k_cache || !v_cache || !slot_mapping)
    return set_error(kInvalid, "kvb_store_kv: NULL pointer");
  if (row % 8 || key_stride % 8 || value_stride % 8 || block_stride % 8 || !aligned16(key) || !aligned16(value) ||
      !aligned16(k_cache) || !aligned16(v_cache))
    return set_error(kInvalid, "kvb_store_kv: rows and strides must be 16-byte aligned");
  if (block_stride < (int64_t)block_size * row)
    return set_error(kInvalid, "kvb_store_kv: block_stride smaller than one block");
  return cuda_status(launch_kernel(store_kv_kernel, dim3(blocks_for(num_tokens, 8)), dim3(256), 0, (cudaStream_t)stream,
                                   (const bf16*)key, key_stride, (const bf16*)value, value_stride, (bf16*)k_cache,
                                   (bf16*)v_cache, num_blocks * block_size, block_stride, block_size, row, slot_mapping,
                                   num_tokens),
                     "kvb_store_kv launch");
}

extern "C" int kvb_rmsnorm(const void* x, int64_t x_stride_t, int64_t x_stride_h, void* out, int64_t out_stride_t,
                           int64_t out_stride_h, const void* weight, int tokens, int heads, int n_cols, float eps,
                           void* stream) {
  if (tokens < 0 || heads <= 0 || n_cols <= 0) return set_error(kInvalid, "kvb_rmsnorm: bad sizes");
  if (tokens == 0) return kOk;
  if (!x || !out || !weight) return set_error(kInvalid, "kvb_rmsnorm: NULL pointer");
  const int64_t rows = (int64_t)tokens * heads;
  if (rows > INT32_MAX) return set_error(kUnsupported, "kvb_rmsnorm: too many rows");
  if (n_cols == 128 && x_stride_t % 4 == 0 && x_stride_h % 4 == 0 && out_stride_t % 4 == 0 &&
      out_stride_h % 4 == 0 && ((uintptr_t)x & 7) == 0 && ((uintptr_t)out & 7) == 0 && ((uintptr_t)weight & 7) == 0) {
    return cuda_status(launch_kernel(rmsnorm128_kernel, dim3(blocks_for(rows, 8)), dim3(256), 0, (cudaStream_t)stream,
                                     (const bf16*)x, x_stride_t, x_stride_h, (bf16*)out, out_stride_t, out_stride_h,
                                     (const bf16*)weight, tokens, heads, eps),
                       "kvb_rmsnorm launch");
  }
  if (n_cols % 8 || x_stride_t % 8 || x_stride_h % 8 || out_stride_t % 8 || out_stride_h % 8 || !aligned16(x) ||
      !aligned16(out) || !aligned16(weight))
    return set_error(kInvalid, "kvb_rmsnorm: rows must be 16-byte aligned (n_cols and strides multiples of 8)");
  if (n_cols > kRowThreads * kRowMaxChunks * 8) return set_error(kUnsupported, "kvb_rmsnorm: n_cols > 16384");
  return cuda_status(launch_kernel(rmsnorm_row_kernel, dim3((unsigned)rows), dim3(kRowThreads), 0, (cudaStream_t)stream,
                                   (const bf16*)x, x_stride_t, x_stride_h, (bf16*)out, out_stride_t, out_stride_h,
                                   (const bf16*)weight, heads, n_cols, eps),
                     "kvb_rmsnorm launch");
}

extern "C" int kvb_add_rmsnorm(const void* x, void* residual, void* out, const void* weight, int tokens, int n_cols,
                               float eps, void* stream) {
  if (tokens < 0 || n_cols <= 0) return set_error(kInvalid, "kvb_add_rmsnorm: bad sizes");
  if (tokens == 0) return kOk;
  if (!x || !residual || !out || !weight) return set_error(kInvalid, "kvb_add_rmsnorm: NULL pointer");
  if (n_cols % 8 || !aligned16(x) || !aligned16(residual) || !aligned16(out) || !aligned16(weight))
    return set_error(kInvalid, "kvb_add_rmsnorm: rows must be 16-byte aligned");
  if (n_cols > kRowThreads * kRowMaxChunks * 8) return set_error(kUnsupported, "kvb_add_rmsnorm: n_cols > 16384");
  return cuda_status(launch_kernel(add_rmsnorm_kernel, dim3((unsigned)tokens), dim3(kRowThreads), 0,
                                   (cudaStream_t)stream, (const bf16*)x, (bf16*)residual, (bf16*)out,
                                   (const bf16*)weight, n_cols, eps),
                     "kvb_add_rmsnorm launch");
}

extern "C" int kvb_rope(void* q, int64_t q_stride_t, int64_t q_stride_h, void* k, int64_t k_stride_t,
                        int64_t k_stride_h, const int64_t* positions, const float* cos_sin, int64_t max_position,
                        int tokens, int q_heads, int k_heads, int head_dim, int interleaved, void* stream) {
  if (tokens < 0 || q_heads < 0 || k_heads < 0 || head_dim <= 0 || head_dim % 2 || max_position <= 0)
    return set_error(kInvalid, "kvb_rope: bad sizes");
  if (tokens == 0 || q_heads + k_heads == 0) return kOk;
  if (!positions || !cos_sin || (q_heads && !q) || (k_heads && !k)) return set_error(kInvalid, "kvb_rope: NULL pointer");
  const int64_t rows = (int64_t)tokens * (q_heads + k_heads);
  return cuda_status(launch_kernel(rope_kernel, dim3(blocks_for(rows, 8)), dim3(256), 0, (cudaStream_t)stream, (bf16*)q,
                                   q_stride_t, q_stride_h, (bf16*)k, k_stride_t, k_stride_h, positions, cos_sin,
                                   max_position, tokens, q_heads, k_heads, head_dim, interleaved),
                     "kvb_rope launch");
}

extern "C" int kvb_qknorm_rope_store(void* qkv, int64_t qkv_stride, int tokens, int num_q_heads, int num_kv_heads,
                                     int head_dim, const void* q_weight, const void* k_weight, float eps,
                                     int apply_norm, const int64_t* positions, const float* cos_sin,
                                     int64_t max_position, int interleaved, void* k_cache, void* v_cache,
                                     int64_t num_blocks, int64_t block_stride, int block_size,
                                     const int32_t* slot_mapping, void* stream) {
  if (tokens < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || max_position <= 0)
    return set_error(kInvalid, "kvb_qknorm_rope_store: bad sizes");
  if (head_dim != 128) return set_error(kUnsupported, "kvb_qknorm_rope_store: head_dim must be 128");
  if (tokens == 0) return kOk;
  if (!qkv || !positions || !cos_sin || (apply_norm && (!q_weight || !k_weight)))
    return set_error(kInvalid, "kvb_qknorm_rope_store: NULL pointer");
  if (qkv_stride < (int64_t)(num_q_heads + 2 * num_kv_heads) * 128 || qkv_stride % 4 || ((uintptr_t)qkv & 7))
    return set_error(kInvalid, "kvb_qknorm_rope_store: qkv rows must be 8-byte aligned and hold all heads");
  if (k_cache) {
    if (!v_cache || !slot_mapping || block_size <= 0 || num_blocks < 0 || block_stride % 4 ||
        ((uintptr_t)k_cache & 7) || ((uintptr_t)v_cache & 7) ||
        block_stride < (int64_t)block_size * num_kv_heads * 128)
      return set_error(kInvalid, "kvb_qknorm_rope_store: bad cache arguments");
  }
  const int64_t rows = (int64_t)tokens * (num_q_heads + 2 * num_kv_heads);
  return cuda_status(launch_kernel(qknorm_rope_store_kernel, dim3(blocks_for(rows, 8)), dim3(256), 0,
                                   (cudaStream_t)stream, (bf16*)qkv, qkv_stride, tokens, num_q_heads, num_kv_heads,
                                   (const bf16*)q_weight, (const bf16*)k_weight, eps, apply_norm, positions, cos_sin,
                                   max_position, interleaved, (bf16*)k_cache, (bf16*)v_cache,
                                   num_blocks * (int64_t)block_size, block_stride, block_size, slot_mapping),
                     "kvb_qknorm_rope_store launch");
}

extern "C" int kvb_silu_mul(const void* x, int64_t x_stride, void* out, int64_t out_stride, int tokens, int inter,
                            void* stream) {
  if (tokens < 0 || inter <= 0) return set_error(kInvalid, "kvb_silu_mul: bad sizes");
  if (tokens == 0) return kOk;
  if (!x || !out) return set_error(kInvalid, "kvb_silu_mul: NULL pointer");
  if (inter % 8 || x_stride % 8 || out_stride % 8 || !aligned16(x) || !aligned16(out) || x_stride < 2 * (int64_t)inter)
    return set_error(kInvalid, "kvb_silu_mul: rows must be 16-byte aligned");
  const int64_t total = (int64_t)tokens * (inter / 8);
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  return cuda_status(launch_kernel(silu_mul_kernel, dim3((unsigned)blocks), dim3(256), 0, (cudaStream_t)stream,
                                   (const bf16*)x, x_stride, (bf16*)out, out_stride, tokens, inter),
                     "kvb_silu_mul launch");
}

extern "C" int kvb_embedding(const int64_t* ids, const void* weight, void* out, int tokens, int hidden,
                             int64_t vocab_start, int64_t vocab_end, int64_t vocab_size, void* stream) {
  if (tokens < 0 || hidden <= 0 || vocab_end < vocab_start) return set_error(kInvalid, "kvb_embedding: bad sizes");
  if (tokens == 0) return kOk;
  if (!ids || !weight || !out) return set_error(kInvalid, "kvb_embedding: NULL pointer");
  if (hidden % 8 || !aligned16(weight) || !aligned16(out))
    return set_error(kInvalid, "kvb_embedding: rows must be 16-byte aligned");
  return cuda_status(launch_kernel(embedding_kernel, dim3((unsigned)tokens), dim3(128), 0, (cudaStream_t)stream, ids,
                                   (const bf16*)weight, (bf16*)out, hidden, vocab_start, vocab_end, vocab_size),
                     "kvb_embedding launch");
}
