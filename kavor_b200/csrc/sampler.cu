// Token sampler (sampler.py:7-66): token = argmax_v(logit[v] / T + Gumbel(v)),
// greedy argmax when T == 0, ties resolved to the lowest index like
// torch.argmax. One CTA per row streams the vocabulary with 16-byte loads.
//
// Noise: Philox4x32-10 counter-based generator (Salmon, Moraes, Dror, Shaw,
// "Parallel random numbers: as easy as 1, 2, 3", SC'11), key = (seed, 0),
// counter = (global column index of the row-major [batch, vocab] matrix) / 4;
// each call yields the uniforms of 4 consecutive columns. The counter uses the
// GLOBAL column, so a vocab-sharded run (kvb_sample_partial on every rank +
// kvb_sample_combine) draws exactly the noise the single-GPU run draws.
#include "common.cuh"
#include "../../include/kavor_b200.h"

KVB_DEFINE_ERROR_WORD(sampler)

namespace kvb {
namespace {

constexpr int kThreads = 512;

__device__ __forceinline__ void philox4x32_10(uint32_t c0, uint32_t c1, uint32_t k0, uint32_t k1, uint32_t out[4]) {
  uint32_t c[4] = {c0, c1, 0u, 0u};
  // multipliers and Weyl key increments of Philox4x32 (SC'11, Table 2 / sec. 3.3)
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u, W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(M0, c[0]), lo0 = M0 * c[0];
    const uint32_t hi1 = __umulhi(M1, c[2]), lo1 = M1 * c[2];
    const uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
    c[0] = n0;
    c[1] = lo1;
    c[2] = n2;
    c[3] = lo0;
    k0 += W0;
    k1 += W1;
  }
  out[0] = c[0];
  out[1] = c[1];
  out[2] = c[2];
  out[3] = c[3];
}

// Uniform in the open interval (0, 1) from the top 23 bits: (k + 0.5) / 2^23
// is exact in fp32 for every k < 2^23, so u never rounds to 0 or 1.
__device__ __forceinline__ float to_unit(uint32_t x) { return ((float)(x >> 9) + 0.5f) * (1.0f / 8388608.0f); }

struct Best {
  float v;
  int64_t i;
};

__device__ __forceinline__ void take(Best& b, float v, int64_t i) {
  if (v > b.v || (v == b.v && i < b.i)) {
    b.v = v;
    b.i = i;
  }
}

__device__ __forceinline__ Best block_argmax(Best b) {
  __shared__ float sv[kThreads / 32];
  __shared__ int64_t si[kThreads / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float v = __shfl_xor_sync(0xffffffffu, b.v, o);
    const int64_t i = __shfl_xor_sync(0xffffffffu, b.i, o);
    take(b, v, i);
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    sv[w] = b.v;
    si[w] = b.i;
  }
  __syncthreads();
  if (w == 0) {
    b.v = l < kThreads / 32 ? sv[l] : -INFINITY;
    b.i = l < kThreads / 32 ? si[l] : INT64_MAX;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float v = __shfl_xor_sync(0xffffffffu, b.v, o);
      const int64_t i = __shfl_xor_sync(0xffffffffu, b.i, o);
      take(b, v, i);
    }
  }
  return b;
}

// Largest Gumbel value the generator can produce: u <= 1 - 2^-24, so
// -log(-log(u)) <= -log(2^-24) = 24 ln 2 = 16.64 (plus margin for logf).
constexpr float kGumbelMax = 16.7f;

__device__ __forceinline__ float gumbel_of(uint32_t r) { return -logf(-logf(to_unit(r))); }

__device__ __forceinline__ float gumbel_at(uint64_t n, uint32_t seed) {
  uint32_t r[4];
  philox4x32_10((uint32_t)(n >> 2), (uint32_t)(n >> 34), seed, 0u, r);
  return gumbel_of(r[n & 3]);
}

// Scores one row segment [0, n) whose column j has global index gcol0 + j in a
// row of vocab_total columns; returns the (score, global index) maximum.
// With T > 0 it runs two passes: (1) the largest logit and its lowest index
// j*, giving the lower bound L = logit[j*] / T + g(j*) of the winning score;
// (2) noise only for columns with logit / T >= L - kGumbelMax — every other
// column's best possible score is below L, so skipping it cannot change the
// result (exact, not an approximation).
__device__ Best score_segment(const bf16* __restrict__ row, int n, int64_t gcol0, int64_t row_base, float temp,
                              uint32_t seed, bool vec) {
  Best best = {-INFINITY, INT64_MAX};
  const int nv = vec ? n / 8 : 0;
  // pass 1 (also the whole greedy path): largest logit, lowest index on ties
  for (int c = threadIdx.x; c < nv; c += kThreads) {
    const uint4 raw = reinterpret_cast<const uint4*>(row)[c];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 p = __bfloat1622float2(h[j]);
      take(best, p.x, gcol0 + c * 8 + 2 * j);
      take(best, p.y, gcol0 + c * 8 + 2 * j + 1);
    }
  }
  for (int j = nv * 8 + threadIdx.x; j < n; j += kThreads) take(best, __bfloat162float(row[j]), gcol0 + j);
  if (!(temp > 0.f)) return best;
  const float inv_t = 1.f / temp;
  best = block_argmax(best);
  __shared__ float bound_s;
  if (threadIdx.x == 0)
    bound_s = best.i == INT64_MAX ? -INFINITY
                                  : best.v * inv_t + gumbel_at((uint64_t)(row_base + best.i), seed) - kGumbelMax;
  __syncthreads();
  const float bound = bound_s;
  best = {-INFINITY, INT64_MAX};
  // pass 2: noise for the candidates only. One Philox block gives the noise
  // of 4 consecutive global columns (counter n / 4, lane n % 4): when the
  // 8 columns of a 16-byte chunk start at a multiple of 4, two blocks serve
  // all 8 instead of one block per column (the same values either way).
  for (int c = threadIdx.x; c < nv; c += kThreads) {
    const uint4 raw = reinterpret_cast<const uint4*>(row)[c];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
    float l[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 p = __bfloat1622float2(h[j]);
      l[2 * j] = p.x * inv_t;
      l[2 * j + 1] = p.y * inv_t;
    }
    const int64_t g0 = gcol0 + c * 8;
    const uint64_t n0 = (uint64_t)(row_base + g0);
    if ((n0 & 3) == 0) {
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        bool any = false;
#pragma unroll
        for (int k = 0; k < 4; ++k) any |= l[4 * q + k] >= bound;
        if (!any) continue;
        const uint64_t n = n0 + 4 * q;
        uint32_t r[4];
        philox4x32_10((uint32_t)(n >> 2), (uint32_t)(n >> 34), seed, 0u, r);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if (l[4 * q + k] >= bound) take(best, l[4 * q + k] + gumbel_of(r[k]), g0 + 4 * q + k);
      }
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (l[k] >= bound) take(best, l[k] + gumbel_at(n0 + k, seed), g0 + k);
    }
  }
  for (int j = nv * 8 + threadIdx.x; j < n; j += kThreads) {
    const float l = __bfloat162float(row[j]) * inv_t;
    if (l >= bound) take(best, l + gumbel_at((uint64_t)(row_base + gcol0 + j), seed), gcol0 + j);
  }
  return best;
}

__global__ void __launch_bounds__(kThreads) sample_kernel(const bf16* __restrict__ logits, int64_t row_stride,
                                                          const float* __restrict__ temps,
                                                          const int32_t* __restrict__ seed, int64_t* __restrict__ out,
                                                          int vocab, bool vec) {
  kernel_entry();
  const int b = blockIdx.x;
  Best best = score_segment(logits + (int64_t)b * row_stride, vocab, 0, (int64_t)b * vocab, temps[b],
                            (uint32_t)seed[0], vec);
  best = block_argmax(best);
  if (threadIdx.x == 0) out[b] = best.i == INT64_MAX ? 0 : best.i;
}

__global__ void __launch_bounds__(kThreads) sample_partial_kernel(const bf16* __restrict__ logits, int64_t row_stride,
                                                                  const float* __restrict__ temps,
                                                                  const int32_t* __restrict__ seed,
                                                                  float* __restrict__ best_val,
                                                                  int64_t* __restrict__ best_idx, int shard_vocab,
                                                                  int64_t vocab_offset, int64_t vocab_total, bool vec) {
  kernel_entry();
  const int b = blockIdx.x;
  Best best = score_segment(logits + (int64_t)b * row_stride, shard_vocab, vocab_offset, (int64_t)b * vocab_total,
                            temps[b], (uint32_t)seed[0], vec);
  best = block_argmax(best);
  if (threadIdx.x == 0) {
    best_val[b] = best.v;
    best_idx[b] = best.i == INT64_MAX ? -1 : best.i;
  }
}

__global__ void sample_combine_kernel(const float* __restrict__ vals, const int64_t* __restrict__ idxs, int world,
                                      int64_t* __restrict__ out, int batch) {
  kernel_entry();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  Best best = {-INFINITY, INT64_MAX};
  for (int r = 0; r < world; ++r) {
    const int64_t i = idxs[(int64_t)r * batch + b];
    if (i >= 0) take(best, vals[(int64_t)r * batch + b], i);
  }
  out[b] = best.i == INT64_MAX ? 0 : best.i;
}

}  // namespace
}  // namespace kvb

using namespace kvb;

extern "C" int kvb_sample(const void* logits, int64_t row_stride, const float* temperatures, const int32_t* seed,
                          int64_t* out, int batch, int vocab, void* stream) {
  if (batch < 0 || vocab <= 0 || row_stride < vocab) return set_error(kInvalid, "kvb_sample: bad sizes");
  if (batch == 0) return kOk;
  if (!logits || !temperatures || !seed || !out) return set_error(kInvalid, "kvb_sample: NULL pointer");
  const bool vec = ((uintptr_t)logits & 15) == 0 && row_stride % 8 == 0;
  return cuda_status(launch_kernel(sample_kernel, dim3(batch), dim3(kThreads), 0, (cudaStream_t)stream,
                                   (const bf16*)logits, row_stride, temperatures, seed, out, vocab, vec),
                     "kvb_sample launch");
}

extern "C" int kvb_sample_partial(const void* logits, int64_t row_stride, const float* temperatures,
                                  const int32_t* seed, float* best_val, int64_t* best_idx, int batch, int shard_vocab,
                                  int64_t vocab_offset, int64_t vocab_total, void* stream) {
  if (batch < 0 || shard_vocab <= 0 || row_stride < shard_vocab || vocab_offset < 0 ||
      vocab_offset + shard_vocab > vocab_total)
    return set_error(kInvalid, "kvb_sample_partial: bad sizes");
  if (batch == 0) return kOk;
  if (!logits || !temperatures || !seed || !best_val || !best_idx)
    return set_error(kInvalid, "kvb_sample_partial: NULL pointer");
  const bool vec = ((uintptr_t)logits & 15) == 0 && row_stride % 8 == 0;
  return cuda_status(launch_kernel(sample_partial_kernel, dim3(batch), dim3(kThreads), 0, (cudaStream_t)stream,
                                   (const bf16*)logits, row_stride, temperatures, seed, best_val, best_idx, shard_vocab,
                                   vocab_offset, vocab_total, vec),
                     "kvb_sample_partial launch");
}

extern "C" int kvb_sample_combine(const float* vals, const int64_t* idxs, int world_size, int64_t* out, int batch,
                                  void* stream) {
  if (batch < 0 || world_size <= 0) return set_error(kInvalid, "kvb_sample_combine: bad sizes");
  if (batch == 0) return kOk;
  if (!vals || !idxs || !out) return set_error(kInvalid, "kvb_sample_combine: NULL pointer");
  return cuda_status(launch_kernel(sample_combine_kernel, dim3((batch + 127) / 128), dim3(128), 0, (cudaStream_t)stream,
                                   vals, idxs, world_size, out, batch),
                     "kvb_sample_combine launch");
}
