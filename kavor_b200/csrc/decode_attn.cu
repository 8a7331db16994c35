// Single-token decode attention over Kavor's paged KV cache
// (flash_attention_kvcache.py:80-83: flash_attn_with_kvcache with
// cache_seqlens = context_lens, block_table, causal=True, scale head_dim^-0.5).
//
// Design (HBM-bound; the bound is the K/V bytes of every context token):
//   grid  = (num_splits, num_kv_heads, batch). One CTA streams a contiguous
//           range of 64-token tiles of one (sequence, kv head) and serves all
//           G = Hq/Hkv query heads of that kv head (GQA packing), so every K/V
//           byte is read from HBM exactly once.
//   warps = 1 producer warp that issues TMA loads (4-D tensor map over the
//           page pool: [head_dim, kv_head, token_in_block, block]; 128-byte
//           swizzle, L2 evict-first) into a 3-stage mbarrier pipeline, and 4
//           consumer warps that each own 16 tokens of a tile and run
//           S = Q K^T and O += P V on warp-level bf16 MMAs (16 query rows, the
//           G valid ones padded), with an fp32 online softmax per warp.
//   merge = the 4 warps are merged in shared memory; with num_splits > 1 the
//           split results (normalised O + log2-sum-exp) go to the caller's
//           workspace and a second kernel merges them.
// Every mbarrier wait is bounded (common.cuh); a block id outside the pool
// raises the device error bit and the tile is read as zeros (TMA OOB fill).
#include <cudaTypedefs.h>

#include <atomic>

#include "common.cuh"
#include "../../include/kavor_b200.h"

KVB_DEFINE_ERROR_WORD(decode)

namespace kvb {
namespace {

constexpr int kHD = 128;
constexpr int kTile = 64;
constexpr int kStages = 3;
constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kHalfBytes = kTile * 128;       // 64 rows x 64 dims x 2 B
constexpr int kKVBytes = 2 * kHalfBytes;      // one K (or V) tile
constexpr int kStageBytes = 2 * kKVBytes;     // K + V
constexpr int kSmemBytes = kStages * kStageBytes + 1024;
constexpr int kMaxGroup = 8;

struct DecodeArgs {
  const bf16* q;
  int64_t q_st, q_sh;
  bf16* out;
  int64_t o_st, o_sh;
  const int32_t* block_tables;
  int64_t bt_stride;
  int max_blocks;
  const int32_t* context_lens;
  float* part_o;    // [batch, hq, splits, 128]
  float* part_lse;  // [batch, hq, splits]
  int num_blocks;
  int block_size;
  int hq, group, num_splits;
  float scale_log2;
};

__device__ __forceinline__ uint32_t swz(uint32_t base, int row, int chunk) {
  // chunk in [0,16): 16-byte column of a 128-dim row split in two 64-dim halves
  return base + (chunk >> 3) * kHalfBytes + row * 128 + ((((chunk & 7) ^ (row & 7))) << 4);
}

__global__ void __launch_bounds__(kThreads, 2)
    decode_attn_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                       const __grid_constant__ DecodeArgs a) {
  kernel_entry();
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[kStages];
  __shared__ __align__(8) uint64_t empty_bar[kStages];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int ctx = a.context_lens[b];
  if (ctx < 0) ctx = 0;
  const int ntiles = (ctx + kTile - 1) / kTile;
  const int tps = (ntiles + a.num_splits - 1) / a.num_splits;
  const int t_begin = min(split * tps, ntiles);
  const int niter = min(t_begin + tps, ntiles) - t_begin;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), kConsumerWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && niter > 0) {
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
      const uint64_t pol = l2_evict_first_policy();
      int issued = 0;
      for (int it = 0; it < niter; ++it) {
        const int s = it % kStages;
        if (it >= kStages && !mbar_wait(smem_u32(&empty_bar[s]), ((it / kStages) - 1) & 1, &g_err_decode)) break;
        const int tok = (t_begin + it) * kTile;
        const int col = tok / a.block_size, off = tok - col * a.block_size;
        int blk = col < a.max_blocks ? a.block_tables[(int64_t)b * a.bt_stride + col] : -1;
        if (blk < 0 || blk >= a.num_blocks) {
          atomicOr(&g_err_decode, (unsigned)kErrBlockTable);
          blk = a.num_blocks;  // out of the tensor map: TMA fills zeros
        }
        const uint32_t st = smem_u32(smem + s * kStageBytes);
        const uint32_t fb = smem_u32(&full_bar[s]);
        mbar_arrive_expect_tx(fb, kStageBytes);
        tma_load_4d(st, &kmap, 0, kvh, off, blk, fb, pol);
        tma_load_4d(st + kHalfBytes, &kmap, 64, kvh, off, blk, fb, pol);
        tma_load_4d(st + kKVBytes, &vmap, 0, kvh, off, blk, fb, pol);
        tma_load_4d(st + kKVBytes + kHalfBytes, &vmap, 64, kvh, off, blk, fb, pol);
        issued = it + 1;
      }
      // Never leave the CTA with copies in flight: wait (bounded) for the last
      // phase issued into every stage.
      for (int it = issued - 1; it >= 0 && it >= issued - kStages; --it)
        mbar_wait(smem_u32(&full_bar[it % kStages]), (it / kStages) & 1, &g_err_decode);
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int G = a.group;
  const int r = lane >> 2;  // query row of the MMA tile this lane holds (c0/c1)
  uint32_t qa[8][4];
  {
    const bf16* qrow = a.q + (int64_t)b * a.q_st + (int64_t)(kvh * G + (r < G ? r : 0)) * a.q_sh;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const int d = ks * 16 + (lane & 3) * 2;
      qa[ks][0] = r < G ? *reinterpret_cast<const uint32_t*>(qrow + d) : 0u;
      qa[ks][2] = r < G ? *reinterpret_cast<const uint32_t*>(qrow + d + 8) : 0u;
      qa[ks][1] = 0u;
      qa[ks][3] = 0u;
    }
  }
  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;
  const int tok0 = warp * 16;
  bool ok = true;

  for (int it = 0; it < niter; ++it) {
    const int s = it % kStages;
    if (!mbar_wait(smem_u32(&full_bar[s]), (it / kStages) & 1, &g_err_decode)) {
      ok = false;
      break;
    }
    const uint32_t kb = smem_u32(smem + s * kStageBytes);
    const uint32_t vb = kb + kKVBytes;
    const int tile_tok = (t_begin + it) * kTile;

    if (tile_tok + tok0 + 16 > ctx) {
      // Tail tile: rows past the context hold stale cache bytes (possibly
      // NaN/Inf); zero this warp's V rows there so P=0 cannot produce NaN.
      for (int idx = lane; idx < 16 * 16; idx += 32) {
        const int row = tok0 + (idx >> 4), chunk = idx & 15;
        if (tile_tok + row >= ctx)
          asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(swz(vb, row, chunk)), "r"(0u) : "memory");
      }
      __syncwarp();
    }

    float sc[2][4];
#pragma unroll
    for (int j = 0; j < 2; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const int m = lane >> 3;
      const int row = tok0 + (lane & 7) + ((m >> 1) << 3);
      uint32_t b0, b1, b2, b3;
      ldmatrix_x4(swz(kb, row, ks * 2 + (m & 1)), b0, b1, b2, b3);
      mma_bf16_16816(sc[0], qa[ks], b0, b1);
      mma_bf16_16816(sc[1], qa[ks], b2, b3);
    }
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = tile_tok + tok0 + j * 8 + (lane & 3) * 2 + e;
        sc[j][e] = t < ctx ? sc[j][e] * a.scale_log2 : -INFINITY;
        mx = fmaxf(mx, sc[j][e]);
      }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float m_new = fmaxf(m_run, mx);
    const float base = m_new == -INFINITY ? 0.f : m_new;
    const float corr = exp2f(m_run - base);
    float p[2][2];
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 2; ++e) p[j][e] = exp2f(sc[j][e] - base);
    l_run = l_run * corr + (p[0][0] + p[0][1]) + (p[1][0] + p[1][1]);
    m_run = m_new;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      o[n][0] *= corr;
      o[n][1] *= corr;
    }
    const uint32_t pa[4] = {pack_bf16(p[0][0], p[0][1]), 0u, pack_bf16(p[1][0], p[1][1]), 0u};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int m = lane >> 3;
      const int row = tok0 + (lane & 7) + ((m & 1) << 3);
      uint32_t b0, b1, b2, b3;
      ldmatrix_x4_trans(swz(vb, row, 2 * i + (m >> 1)), b0, b1, b2, b3);
      mma_bf16_16816(o[2 * i], pa, b0, b1);
      mma_bf16_16816(o[2 * i + 1], pa, b2, b3);
    }
    // order this warp's generic-proxy smem writes (tail zeroing) before the
    // producer's next async-proxy (TMA) write into the stage
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&empty_bar[s]));
  }

  // ------------------------------------------------ merge the 4 consumer warps
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
  // all copies this CTA issued have landed once every consumer passed its
  // waits; the stage buffers are reused as merge scratch
  named_bar_sync(1, kConsumerWarps * 32);
  float* ow = reinterpret_cast<float*>(smem);                   // [4][8][128]
  float* mw = ow + kConsumerWarps * kMaxGroup * kHD;            // [4][8]
  float* lw = mw + kConsumerWarps * kMaxGroup;                  // [4][8]
  if (!ok) {
    m_run = -INFINITY;
    l_run = 0.f;
  }
  if (r < G) {
    if ((lane & 3) == 0) {
      mw[warp * kMaxGroup + r] = m_run;
      lw[warp * kMaxGroup + r] = l_run;
    }
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      const int d = n * 8 + (lane & 3) * 2;
      ow[(warp * kMaxGroup + r) * kHD + d] = o[n][0];
      ow[(warp * kMaxGroup + r) * kHD + d + 1] = o[n][1];
    }
  }
  named_bar_sync(1, kConsumerWarps * 32);
  for (int idx = threadIdx.x; idx < G * kHD; idx += kConsumerWarps * 32) {
    const int row = idx / kHD, d = idx - row * kHD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, mw[w * kMaxGroup + row]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) {
      const float mv = mw[w * kMaxGroup + row];
      const float f = mv == -INFINITY ? 0.f : exp2f(mv - M);
      L += f * lw[w * kMaxGroup + row];
      O += f * ow[(w * kMaxGroup + row) * kHD + d];
    }
    const int head = kvh * G + row;
    if (a.num_splits == 1) {
      a.out[(int64_t)b * a.o_st + (int64_t)head * a.o_sh + d] = __float2bfloat16_rn(L > 0.f ? O / L : 0.f);
    } else {
      const int64_t pi = ((int64_t)b * a.hq + head) * a.num_splits + split;
      a.part_o[pi * kHD + d] = L > 0.f ? O / L : 0.f;
      if (d == 0) a.part_lse[pi] = L > 0.f ? M + log2f(L) : -INFINITY;
    }
  }
}

// Merge num_splits partial results per (sequence, query head).
__global__ void decode_merge_kernel(const float* __restrict__ part_o, const float* __restrict__ part_lse,
                                    bf16* __restrict__ out, int64_t o_st, int64_t o_sh, int hq, int splits) {
  kernel_entry();
  const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
  const int64_t base = ((int64_t)b * hq + h) * splits;
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, part_lse[base + s]);
  float W = 0.f, O = 0.f;
  if (M != -INFINITY) {
    for (int s = 0; s < splits; ++s) {
      const float l = part_lse[base + s];
      if (l == -INFINITY) continue;
      const float w = exp2f(l - M);
      W += w;
      O += w * part_o[(base + s) * kHD + d];
    }
  }
  out[(int64_t)b * o_st + (int64_t)h * o_sh + d] = __float2bfloat16_rn(W > 0.f ? O / W : 0.f);
}

int encode_kv_map(CUtensorMap* map, const void* base, int64_t num_blocks, int64_t block_stride, int block_size,
                  int hkv) {
  auto enc = tensor_map_encoder();
  if (!enc) return set_error(kNoEncoder, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[4] = {(cuuint64_t)kHD, (cuuint64_t)hkv, (cuuint64_t)block_size, (cuuint64_t)num_blocks};
  const cuuint64_t strides[3] = {(cuuint64_t)kHD * 2, (cuuint64_t)hkv * kHD * 2, (cuuint64_t)block_stride * 2};
  const cuuint32_t box[4] = {64, 1, (cuuint32_t)kTile, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(kEncode, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
  return kOk;
}

// Split the context only when (sequence, kv head) units leave more than half
// of the 2-per-SM CTA slots idle, and then into as many parts as one wave
// holds: at B=256 x 1 kv head (TP=8) one unsplit wave measured 23 us against
// 40 us split three ways (the extra wave, the partial traffic and the merge).
int choose_splits(int batch, int hkv, int max_tiles, int sms) {
  const int units = batch * hkv;
  const int slots = 2 * sms;  // two CTAs fit per SM
  if (2 * units >= slots || max_tiles <= 1) return 1;
  int s = slots / units;
  if (s > max_tiles) s = max_tiles;
  if (s > 64) s = 64;
  return s < 1 ? 1 : s;
}

int current_sms() {
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

int ensure_smem_attr() {
  static unsigned long long done = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
  if (dev < 64 && (done >> dev) & 1ull) return kOk;
  e = cudaFuncSetAttribute(decode_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (e != cudaSuccess) return cuda_status(e, "decode attention smem attribute");
  if (dev < 64) done |= 1ull << dev;
  return kOk;
}

size_t workspace_bytes(int batch, int hq, int splits) {
  if (splits <= 1) return 0;
  const size_t n = (size_t)batch * hq * splits;
  return n * kHD * sizeof(float) + n * sizeof(float);
}

}  // namespace
}  // namespace kvb

using namespace kvb;

extern "C" int kvb_paged_decode_attn_workspace_size(int batch, int num_q_heads, int num_kv_heads, int head_dim,
                                                    int max_blocks_per_seq, int block_size, int num_splits,
                                                    size_t* bytes) {
  if (!bytes) return set_error(kInvalid, "workspace_size: bytes is NULL");
  if (batch < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || head_dim != kHD || max_blocks_per_seq < 0 ||
      block_size <= 0 || num_splits < 0)
    return set_error(kInvalid, "workspace_size: bad sizes");
  const int max_tiles = (int)(((int64_t)max_blocks_per_seq * block_size + kTile - 1) / kTile);
  const int splits = num_splits > 0 ? num_splits : choose_splits(batch, num_kv_heads, max_tiles, current_sms());
  *bytes = workspace_bytes(batch, num_q_heads, splits);
  return kOk;
}

extern "C" int kvb_paged_decode_attn(const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* k_cache,
                                     const void* v_cache, int64_t num_blocks, int64_t block_stride, int block_size,
                                     const int32_t* block_tables, int64_t block_table_stride, int max_blocks_per_seq,
                                     const int32_t* context_lens, void* out, int64_t out_stride_t,
                                     int64_t out_stride_h, int batch, int num_q_heads, int num_kv_heads, int head_dim,
                                     float scale, int num_splits, void* workspace, size_t workspace_bytes_given,
                                     void* stream) {
  if (batch < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads || num_blocks <= 0 ||
      num_blocks >= INT32_MAX || block_size <= 0 || max_blocks_per_seq < 0 || num_splits < 0)
    return set_error(kInvalid, "kvb_paged_decode_attn: bad sizes");
  if (head_dim != kHD) return set_error(kUnsupported, "kvb_paged_decode_attn: head_dim must be 128");
  if (block_size % kTile) return set_error(kUnsupported, "kvb_paged_decode_attn: block_size must be a multiple of 64");
  const int group = num_q_heads / num_kv_heads;
  if (group > kMaxGroup) return set_error(kUnsupported, "kvb_paged_decode_attn: more than 8 query heads per kv head");
  if (batch == 0) return kOk;
  if (!q || !k_cache || !v_cache || !block_tables || !context_lens || !out)
    return set_error(kInvalid, "kvb_paged_decode_attn: NULL pointer");
  if (((uintptr_t)q & 3) || (q_stride_t & 1) || (q_stride_h & 1))
    return set_error(kInvalid, "kvb_paged_decode_attn: q must be 4-byte aligned with even strides");
  if (((uintptr_t)k_cache & 15) || ((uintptr_t)v_cache & 15) || block_stride % 8 ||
      block_stride < (int64_t)block_size * num_kv_heads * kHD)
    return set_error(kInvalid, "kvb_paged_decode_attn: cache must be 16-byte aligned with a full block stride");
  const int max_tiles = (int)(((int64_t)max_blocks_per_seq * block_size + kTile - 1) / kTile);
  const int splits = num_splits > 0 ? num_splits : choose_splits(batch, num_kv_heads, max_tiles, current_sms());
  const size_t need = workspace_bytes(batch, num_q_heads, splits);
  if (need > 0 && (workspace == nullptr || workspace_bytes_given < need))
    return set_error(kWorkspace, "kvb_paged_decode_attn: workspace of %zu bytes needed, %zu given", need,
                     workspace_bytes_given);
  if (need > 0 && ((uintptr_t)workspace & 15)) return set_error(kInvalid, "kvb_paged_decode_attn: workspace alignment");

  CUtensorMap kmap, vmap;
  int rc = encode_kv_map(&kmap, k_cache, num_blocks, block_stride, block_size, num_kv_heads);
  if (rc) return rc;
  rc = encode_kv_map(&vmap, v_cache, num_blocks, block_stride, block_size, num_kv_heads);
  if (rc) return rc;
  rc = ensure_smem_attr();
  if (rc) return rc;

  DecodeArgs a;
  a.q = (const bf16*)q;
  a.q_st = q_stride_t;
  a.q_sh = q_stride_h;
  a.out = (bf16*)out;
  a.o_st = out_stride_t;
  a.o_sh = out_stride_h;
  a.block_tables = block_tables;
  a.bt_stride = block_table_stride;
  a.max_blocks = max_blocks_per_seq;
  a.context_lens = context_lens;
  float* ws = (float*)workspace;
  a.part_o = ws;
  a.part_lse = ws ? ws + (size_t)batch * num_q_heads * splits * kHD : nullptr;
  a.num_blocks = (int)num_blocks;
  a.block_size = block_size;
  a.hq = num_q_heads;
  a.group = group;
  a.num_splits = splits;
  a.scale_log2 = scale * 1.4426950408889634f;

  dim3 grid(splits, num_kv_heads, batch);
  cudaError_t e =
      launch_kernel(decode_attn_kernel, grid, dim3(kThreads), kSmemBytes, (cudaStream_t)stream, kmap, vmap, a);
  if (e != cudaSuccess) return cuda_status(e, "kvb_paged_decode_attn launch");
  if (splits > 1) {
    e = launch_kernel(decode_merge_kernel, dim3(num_q_heads, batch), dim3(kHD), 0, (cudaStream_t)stream,
                      (const float*)a.part_o, (const float*)a.part_lse, (bf16*)out, out_stride_t, out_stride_h,
                      num_q_heads, splits);
    if (e != cudaSuccess) return cuda_status(e, "kvb_paged_decode_attn merge launch");
  }
  return kOk;
}

// ---------------------------------------------------------------------------
// Variant that allocates nothing and takes no scratch pointer.
//
// Some callers cannot hand the library a scratch buffer: their interface only
// carries input and output pointers (a plugin "enqueue" hook, or a binding
// from a host language that has no device allocator), or they run under a
// fixed device-memory budget decided at start-up in which the library may not
// request more memory. For them the split-KV partial results go to this
// built-in area instead of a caller workspace. The area is a file-scope
// device array of kStaticScratchBytes; every GPU that loads the library holds
// it until the process exits. All calls on a device share it: two calls whose
// kernels overlap on the GPU (different streams without ordering) race on it.
// Nothing in it has to start at zero: every split writes all of its partials
// before the merge reads them.
static constexpr size_t kStaticScratchBytes = 8u << 20;  // 8 MiB
static __device__ __align__(256) float g_decode_static_scratch[kStaticScratchBytes / sizeof(float)];

namespace kvb {
namespace {

// Device address of the built-in area for the current device. The lookup runs
// once per device, on the first call made while that device is current (it
// may load the module, which is why that first call belongs before any stream
// capture). The cached address belongs to the device's primary context: a
// process that resets the device (cudaDeviceReset) must not call this entry
// point again. Host threads may race on the first lookup; each stores the same
// address, and the slots are atomic.
int static_scratch_address(float** out) {
  static std::atomic<float*> addr[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "kvb_paged_decode_attn_no_alloc: cudaGetDevice");
  if (dev < 0 || dev >= 64) return set_error(kUnsupported, "kvb_paged_decode_attn_no_alloc: device index >= 64");
  float* p = addr[dev].load(std::memory_order_acquire);
  if (!p) {
    void* sym = nullptr;
    e = cudaGetSymbolAddress(&sym, g_decode_static_scratch);
    if (e != cudaSuccess) return cuda_status(e, "kvb_paged_decode_attn_no_alloc: cudaGetSymbolAddress");
    p = static_cast<float*>(sym);
    addr[dev].store(p, std::memory_order_release);
  }
  *out = p;
  return kOk;
}

}  // namespace
}  // namespace kvb

extern "C" int kvb_paged_decode_attn_no_alloc(const void* q, int64_t q_stride_t, int64_t q_stride_h,
                                              const void* k_cache, const void* v_cache, int64_t num_blocks,
                                              int64_t block_stride, int block_size, const int32_t* block_tables,
                                              int64_t block_table_stride, int max_blocks_per_seq,
                                              const int32_t* context_lens, void* out, int64_t out_stride_t,
                                              int64_t out_stride_h, int batch, int num_q_heads, int num_kv_heads,
                                              int head_dim, float scale, int num_splits, void* stream) {
  if (batch < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads || num_blocks <= 0 ||
      num_blocks >= INT32_MAX || block_size <= 0 || max_blocks_per_seq < 0 || num_splits < 0)
    return set_error(kInvalid, "kvb_paged_decode_attn_no_alloc: bad sizes");
  if (head_dim != kHD) return set_error(kUnsupported, "kvb_paged_decode_attn_no_alloc: head_dim must be 128");
  if (block_size % kTile)
    return set_error(kUnsupported, "kvb_paged_decode_attn_no_alloc: block_size must be a multiple of 64");
  const int group = num_q_heads / num_kv_heads;
  if (group > kMaxGroup)
    return set_error(kUnsupported, "kvb_paged_decode_attn_no_alloc: more than 8 query heads per kv head");
  if (batch == 0) return kOk;
  if (!q || !k_cache || !v_cache || !block_tables || !context_lens || !out)
    return set_error(kInvalid, "kvb_paged_decode_attn_no_alloc: NULL pointer");
  if (((uintptr_t)q & 3) || (q_stride_t & 1) || (q_stride_h & 1))
    return set_error(kInvalid, "kvb_paged_decode_attn_no_alloc: q must be 4-byte aligned with even strides");
  if (((uintptr_t)k_cache & 15) || ((uintptr_t)v_cache & 15) || block_stride % 8 ||
      block_stride < (int64_t)block_size * num_kv_heads * kHD)
    return set_error(kInvalid,
                     "kvb_paged_decode_attn_no_alloc: cache must be 16-byte aligned with a full block stride");
  const int max_tiles = (int)(((int64_t)max_blocks_per_seq * block_size + kTile - 1) / kTile);
  const int splits = num_splits > 0 ? num_splits : choose_splits(batch, num_kv_heads, max_tiles, current_sms());
  const size_t need = workspace_bytes(batch, num_q_heads, splits);
  if (need > kStaticScratchBytes)
    return set_error(kWorkspace,
                     "kvb_paged_decode_attn_no_alloc: %d splits x %d sequences x %d heads need %zu bytes of scratch, "
                     "the built-in area holds %zu; pass fewer splits (1 needs none) or use kvb_paged_decode_attn "
                     "with a caller workspace",
                     splits, batch, num_q_heads, need, kStaticScratchBytes);
  float* ws = nullptr;
  if (need > 0) {
    int rc = static_scratch_address(&ws);
    if (rc) return rc;
  }

  CUtensorMap kmap, vmap;
  int rc = encode_kv_map(&kmap, k_cache, num_blocks, block_stride, block_size, num_kv_heads);
  if (rc) return rc;
  rc = encode_kv_map(&vmap, v_cache, num_blocks, block_stride, block_size, num_kv_heads);
  if (rc) return rc;
  rc = ensure_smem_attr();
  if (rc) return rc;

  DecodeArgs a;
  a.q = (const bf16*)q;
  a.q_st = q_stride_t;
  a.q_sh = q_stride_h;
  a.out = (bf16*)out;
  a.o_st = out_stride_t;
  a.o_sh = out_stride_h;
  a.block_tables = block_tables;
  a.bt_stride = block_table_stride;
  a.max_blocks = max_blocks_per_seq;
  a.context_lens = context_lens;
  a.part_o = ws;
  a.part_lse = ws ? ws + (size_t)batch * num_q_heads * splits * kHD : nullptr;
  a.num_blocks = (int)num_blocks;
  a.block_size = block_size;
  a.hq = num_q_heads;
  a.group = group;
  a.num_splits = splits;
  a.scale_log2 = scale * 1.4426950408889634f;

  dim3 grid(splits, num_kv_heads, batch);
  cudaError_t e =
      launch_kernel(decode_attn_kernel, grid, dim3(kThreads), kSmemBytes, (cudaStream_t)stream, kmap, vmap, a);
  if (e != cudaSuccess) return cuda_status(e, "kvb_paged_decode_attn_no_alloc launch");
  if (splits > 1) {
    e = launch_kernel(decode_merge_kernel, dim3(num_q_heads, batch), dim3(kHD), 0, (cudaStream_t)stream,
                      (const float*)a.part_o, (const float*)a.part_lse, (bf16*)out, out_stride_t, out_stride_h,
                      num_q_heads, splits);
    if (e != cudaSuccess) return cuda_status(e, "kvb_paged_decode_attn_no_alloc merge launch");
  }
  return kOk;
}
