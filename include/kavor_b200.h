/*
 * kavor_b200 — C ABI of the B200 (sm_100a) kernels behind Kavor's Qwen3
 * tensor-parallel decode/prefill path.
 *
 * Conventions shared by every entry point
 *   - Pointers are device pointers unless stated otherwise. Activations and the
 *     KV cache are bf16, metadata is int32 (slot_mapping, block_tables,
 *     context_lens, cu_seqlens) or int64 (token ids, positions), exactly the
 *     dtypes Kavor's ModelRunner builds (model_runner.py:434-473).
 *   - Strides are in ELEMENTS, sizes are element or row counts.
 *   - `stream` is a cudaStream_t passed as void*. Nothing is synchronised and
 *     nothing is allocated inside a call; all of them can be captured in a CUDA
 *     graph. Scratch memory is provided by the caller (query *_workspace_size).
 *   - Return value: 0 = ok, <0 = invalid argument (checked on the host, nothing
 *     launched), >0 = cudaError_t of the launch. kvb_last_error() gives the
 *     message of the calling thread's last failure.
 *   - Paged KV cache layout (cache_pool.py:311-322): one page per block and
 *     layer, K block [block_size, num_kv_heads, head_dim] followed by the V
 *     block; `block_stride` is the element distance between consecutive K
 *     blocks (= 2 * block_size * num_kv_heads * head_dim), v_cache = k_cache +
 *     block_size * num_kv_heads * head_dim.
 */
#ifndef KAVOR_B200_H
#define KAVOR_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* The library is built with hidden visibility; only this API is exported. */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* ------------------------------------------------------------------ library */

/* ABI version (major*10000 + minor*100 + patch). */
int kvb_version(void);

/* Message of the last failed call on this host thread ("" if none). */
const char* kvb_last_error(void);

/* OR of the device-side error bits raised by kernels on the CURRENT device
 * since the last clear (1: block table, 2: slot, 4: wait timeout, 8: token id,
 * 16: peer (all-reduce flag) wait timeout, 32: a launch configuration the
 * kernel cannot serve, its work skipped). Synchronises the device. Returns 0
 * or a CUDA error. */
int kvb_device_error(unsigned* bits, int clear);

/* Launch mode of every later kernel launch from this process on the CURRENT
 * device (no reference counterpart): 1 = programmatic dependent launch (each
 * kernel may be scheduled while the kernel before it on the stream still
 * runs; it waits at its start, griddepcontrol.wait, until that kernel has
 * completed, so results are unchanged), 0 = plain stream-ordered launches
 * (the default). Synchronous (it writes a device constant); call it outside
 * stream capture. */
int kvb_set_pdl(int enable);

/* Number of SMs of the current device (used by the host-side heuristics). */
int kvb_sm_count(int* out);

/* ------------------------------------------------------------ KV-cache write */

/* store_kvcache (flash_attention_kvcache.py:10-46): for every token t with
 * slot_mapping[t] != -1, copy key[t] and value[t] ([num_kv_heads, head_dim],
 * row strides key_stride/value_stride) into block slot/block_size, row
 * slot%block_size of the paged cache. Slots >= num_blocks*block_size raise the
 * device slot error and are skipped. */
int kvb_store_kv(const void* key, int64_t key_stride, const void* value, int64_t value_stride,
                 void* k_cache, void* v_cache, int64_t num_blocks, int64_t block_stride, int block_size,
                 int num_kv_heads, int head_dim, const int32_t* slot_mapping, int num_tokens, void* stream);

/* -------------------------------------------------------------- norms / RoPE */

/* RMSNorm (layernorm.py:8-39, RMSNorm.rms_forward :319-342):
 *   out = bf16( bf16(x * rsqrt(mean(x^2) + eps)) * weight ), fp32 inside.
 * x/out are [tokens, heads, n_cols] with arbitrary token/head strides (heads=1
 * with stride_h ignored for 2-D inputs); the last dimension is contiguous. */
int kvb_rmsnorm(const void* x, int64_t x_stride_t, int64_t x_stride_h, void* out, int64_t out_stride_t,
                int64_t out_stride_h, const void* weight, int tokens, int heads, int n_cols, float eps,
                void* stream);

/* Fused residual add + RMSNorm (layernorm.py:114-140, add_rms_forward :344-372):
 *   r = fp32(x) + fp32(residual); residual <- bf16(r) (in place);
 *   out = bf16( bf16(r * rsqrt(mean(r^2) + eps)) * weight ).
 * x, residual, out are contiguous [tokens, n_cols]. out may alias x. */
int kvb_add_rmsnorm(const void* x, void* residual, void* out, const void* weight, int tokens, int n_cols,
                    float eps, void* stream);

/* In-place rotary embedding of q and k (rotary_embedding.py:8-53, :104-120).
 * cos_sin is the fp32 [max_position, head_dim] table [cos | sin] built as in
 * rotary_embedding.py:96-102; interleaved selects (2i, 2i+1) pairs instead of
 * (i, i + head_dim/2). Positions outside [0, max_position) are clamped and
 * raise no error (the reference does not check them either). */
int kvb_rope(void* q, int64_t q_stride_t, int64_t q_stride_h, void* k, int64_t k_stride_t,
             int64_t k_stride_h, const int64_t* positions, const float* cos_sin, int64_t max_position,
             int tokens, int q_heads, int k_heads, int head_dim, int interleaved, void* stream);

/* Fused Qwen3 attention prologue (qwen3.py:80-89 + flash_attention_kvcache.py:72):
 * on the packed qkv rows [tokens, (Hq + 2*Hkv) * head_dim] (row stride
 * qkv_stride), in place: q_norm and k_norm (RMSNorm over head_dim, weights
 * q_weight/k_weight), RoPE on q and k, then the k and v rows are written into
 * the paged cache at slot_mapping (skipped for -1). apply_norm = 0 skips the
 * norms (attention_bias models); k_cache = NULL skips the cache write. */
int kvb_qknorm_rope_store(void* qkv, int64_t qkv_stride, int tokens, int num_q_heads, int num_kv_heads,
                          int head_dim, const void* q_weight, const void* k_weight, float eps, int apply_norm,
                          const int64_t* positions, const float* cos_sin, int64_t max_position, int interleaved,
                          void* k_cache, void* v_cache, int64_t num_blocks, int64_t block_stride,
                          int block_size, const int32_t* slot_mapping, void* stream);

/* -------------------------------------------------------------- activation */

/* SiluAndMul (activation.py:8-11): out[t, i] = bf16(silu(x[t, i]) * x[t, inter + i]),
 * fp32 inside, one rounding. */
int kvb_silu_mul(const void* x, int64_t x_stride, void* out, int64_t out_stride, int tokens, int inter,
                 void* stream);

/* ---------------------------------------------------------------- embedding */

/* VocabParallelEmbedding lookup (embed_head.py:34-42 without the all-reduce):
 * out[t] = weight[ids[t] - vocab_start] if vocab_start <= ids[t] < vocab_end,
 * else zeros. weight is [vocab_end - vocab_start, hidden], out [tokens, hidden].
 * vocab_size > 0 raises the device token-id error for ids outside [0, vocab_size). */
int kvb_embedding(const int64_t* ids, const void* weight, void* out, int tokens, int hidden, int64_t vocab_start,
                  int64_t vocab_end, int64_t vocab_size, void* stream);

/* ---------------------------------------------------------------- attention */

/* Bytes of scratch kvb_paged_decode_attn needs for this shape and split count
 * (num_splits = 0 means the heuristic the call itself would pick). */
int kvb_paged_decode_attn_workspace_size(int batch, int num_q_heads, int num_kv_heads, int head_dim,
                                         int max_blocks_per_seq, int block_size, int num_splits,
                                         size_t* bytes);

/* Single-token decode attention over the paged cache
 * (flash_attention_kvcache.py:80-83 = flash_attn_with_kvcache(q.unsqueeze(1),
 * k_cache, v_cache, cache_seqlens=context_lens, block_table, causal=True)).
 * q/out are [batch, num_q_heads, head_dim]; query head h reads kv head
 * h / (num_q_heads / num_kv_heads). Rows with context_lens = 0 produce zeros.
 * K/V blocks are staged into shared memory with TMA; the context is split
 * across CTAs (num_splits; 0 = heuristic) and merged in a second kernel
 * through `workspace` (>= kvb_paged_decode_attn_workspace_size bytes). */
int kvb_paged_decode_attn(const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* k_cache,
                          const void* v_cache, int64_t num_blocks, int64_t block_stride, int block_size,
                          const int32_t* block_tables, int64_t block_table_stride, int max_blocks_per_seq,
                          const int32_t* context_lens, void* out, int64_t out_stride_t, int64_t out_stride_h,
                          int batch, int num_q_heads, int num_kv_heads, int head_dim, float scale,
                          int num_splits, void* workspace, size_t workspace_bytes, void* stream);

/* No counterpart in the reference. The same decode attention for callers that
 * cannot provide scratch memory: their interface passes only inputs and
 * outputs (a plugin enqueue hook, a binding from a host language without a
 * device allocator), or their device-memory budget is fixed at start-up. It
 * allocates nothing: split-KV partials go to a built-in 8 MiB device array
 * that every GPU loading the library keeps until the process exits. The first
 * call on each device looks up that array's address (make that first call
 * before any stream capture). Shapes whose partials would exceed 8 MiB
 * (batch x num_q_heads x splits x 516 bytes) are rejected with kWorkspace (-3);
 * num_splits = 1 needs no scratch. All calls on a device share the array, so
 * calls whose kernels overlap on the GPU (unordered streams) race. */
int kvb_paged_decode_attn_no_alloc(const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* k_cache,
                                   const void* v_cache, int64_t num_blocks, int64_t block_stride, int block_size,
                                   const int32_t* block_tables, int64_t block_table_stride, int max_blocks_per_seq,
                                   const int32_t* context_lens, void* out, int64_t out_stride_t, int64_t out_stride_h,
                                   int batch, int num_q_heads, int num_kv_heads, int head_dim, float scale,
                                   int num_splits, void* stream);

/* Causal varlen prefill attention (flash_attention_kvcache.py:73-79 =
 * flash_attn_varlen_func(..., causal=True, block_table)). Sequence b owns
 * queries [cu_seqlens_q[b], cu_seqlens_q[b+1]) and attends keys
 * [0, cu_seqlens_k[b+1] - cu_seqlens_k[b]) with bottom-right causal alignment.
 * Keys come from the paged cache through block_tables (prefix cache / chunked
 * prefill) when block_tables != NULL, else from the contiguous k/v rows
 * [cu_seqlens_k[b] + j] (k_stride_t/h, v_stride_t/h). q/out [total_q, Hq, hd].
 * total_q (rows of q) and total_k (rows of the contiguous k/v; unused when
 * paged) bound the kernel's TMA maps: with them, page sizes that are a
 * multiple of 128 and 16-byte output rows, QK^T and PV run on tcgen05 with
 * TMEM accumulators; with total_q = 0 (or other page sizes) the warp-MMA
 * kernel runs instead. */
int kvb_prefill_attn(const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* k, int64_t k_stride_t,
                     int64_t k_stride_h, const void* v, int64_t v_stride_t, int64_t v_stride_h,
                     int64_t num_blocks, int64_t block_stride, int block_size, const int32_t* block_tables,
                     int64_t block_table_stride, int max_blocks_per_seq, const int32_t* cu_seqlens_q,
                     const int32_t* cu_seqlens_k, int batch, int max_seqlen_q, void* out, int64_t out_stride_t,
                     int64_t out_stride_h, int num_q_heads, int num_kv_heads, int head_dim, float scale,
                     int64_t total_q, int64_t total_k, void* stream);

/* --------------------------------------------------------------------- GEMM */

/* Bytes of scratch kvb_gemm_bf16 needs for this shape: always 0 (a K split
 * reduces through distributed shared memory); kept so callers can size and
 * pass a workspace uniformly. */
int kvb_gemm_workspace_size(int M, int N, int K, int splits, size_t* bytes);

/* y[M, N] = x[M, K] * w[N, K]^T (F.linear of linear.py:50,73,157 and
 * embed_head.py:61) on tcgen05 tensor cores: bf16 operands, fp32 accumulation
 * in TMEM, bf16 result; rows of x, w, y with leading dimensions ldx, ldw, ldy
 * (elements; x and w rows 16-byte aligned). The weight is streamed once per
 * token tile (up to 256 tokens) through TMA. splits = 0 lets a cost model
 * pick the token tile and the K split (among 1, 2, 4, 8, 16); splits in 1..16
 * asks for that split (a thread-block cluster of that many CTAs whose fp32
 * parts are summed in a fixed order through distributed shared memory:
 * deterministic), falling back to the cost model's choice when no token tile
 * can take it (more CTAs than K-steps, or a reduction that does not fit the
 * CTA's shared memory). `workspace` is unused (may be NULL). */
int kvb_gemm_bf16(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy, int M, int N, int K,
                  int splits, void* workspace, size_t workspace_bytes, void* stream);

/* Gate-up projection fused with SiluAndMul (linear.py:76-93 + activation.py:8-11):
 * w is the [2 * inter, K] merged weight with rows [gate | up];
 * y[M, inter] = bf16( silu(bf16(x w_gate^T)) * bf16(x w_up^T) ), fp32 inside —
 * the reference's rounding points, without the [M, 2*inter] intermediate.
 * Split and workspace rules as kvb_gemm_bf16. */
int kvb_gemm_silu_workspace_size(int M, int inter, int K, int splits, size_t* bytes);
int kvb_gemm_silu_bf16(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy, int M, int inter,
                       int K, int splits, void* workspace, size_t workspace_bytes, void* stream);

/* The tiling the GEMM picks for this shape on the current device (N = output
 * width; gated = the fused SiLU form): plan[0] token tile, plan[1] K splits,
 * plan[2] work units, plan[3] CTAs. */
int kvb_gemm_plan(int M, int N, int K, int splits, int gated, int* plan);

/* y[M, N] = x[M, K] * w[N, K]^T on CTA pairs (tcgen05 cta_group::2; no
 * reference counterpart beyond the F.linear it computes): each pair of a
 * thread-block cluster multiplies 256 weight rows (128 per CTA) by a token
 * tile of 64, 128 or 256 tokens (half per CTA) with one MMA per 16-wide K
 * step, and `splits` pairs (1..8, 0 = chosen for one CTA per SM) share K
 * through a distributed-shared-memory reduction in a fixed order. Same
 * operand rules as kvb_gemm_bf16; no workspace. */
int kvb_gemm_pair_bf16(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy, int M, int N,
                       int K, int splits, void* stream);
/* Gate-up projection fused with SiluAndMul on CTA pairs: w is the [2 * inter,
 * K] merged weight with rows [gate | up]; the even CTA of each pair holds 128
 * gate rows, the odd CTA the up rows of the same features, and
 * y[M, inter] = bf16(silu(bf16(x w_gate^T)) * bf16(x w_up^T)). K split as
 * kvb_gemm_pair_bf16 (0 = planned). */
int kvb_gemm_pair_silu_bf16(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy, int M,
                            int inter, int K, int splits, void* stream);
/* The pair GEMM's plan for this shape (host only; gated: N = inter, the
 * fused SiLU form): plan[0] token tile, plan[1] K splits, plan[2] tiles,
 * plan[3] CTAs. */
int kvb_gemm_pair_plan(int M, int N, int K, int splits, int gated, int* plan);

/* Decode-batch GEMM (the F.linear of linear.py:50,73,157 and embed_head.py:61
 * at M <= 256 tokens; larger M works, tiled by 256 tokens): y[M, N] =
 * x[M, K] * w[N, K]^T on CTA pairs (tcgen05 cta_group::2, 256 weight rows x up
 * to 256 tokens per MMA) with a stream-K schedule: one wave of persistent
 * pairs shares the (tile, K-step) iterations equally; a tile cut between
 * pairs is summed by its first segment from fp32 partials the others leave in
 * `workspace`, in K order (deterministic). Operand rules as kvb_gemm_bf16.
 * `workspace` (256-byte aligned, at least kvb_gemm_sk_workspace_size bytes)
 * must be zero when first used; the kernel leaves it zero again after every
 * normal launch (after a device error bit it must be zeroed again). Launches
 * that share a workspace must be ordered on one stream. */
int kvb_gemm_sk_workspace_size(int M, int N, int K, int gated, size_t* bytes);
int kvb_gemm_sk_bf16(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy, int M, int N, int K,
                     void* workspace, size_t workspace_bytes, void* stream);
/* Gate-up projection fused with SiluAndMul (linear.py:76-93 + activation.py:8-11)
 * on the same schedule: w is the [2 * inter, K] merged weight with rows
 * [gate | up]; each CTA multiplies 64 gate rows and the same features' 64 up
 * rows; y[M, inter] = bf16(silu(bf16(x w_gate^T)) * bf16(x w_up^T)). */
int kvb_gemm_sk_silu_bf16(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy, int M,
                          int inter, int K, void* workspace, size_t workspace_bytes, void* stream);
/* The stream-K GEMM's plan for this shape (host only; gated: N = inter):
 * plan[0] token tile, plan[1] tiles, plan[2] K-steps per tile, plan[3] pairs
 * (at most half the SMs; a launch may use fewer when fewer 2-CTA clusters fit). */
int kvb_gemm_sk_plan(int M, int N, int K, int gated, int* plan);

/* Process-wide tuning of the stream-K GEMM (no reference counterpart): force
 * the token tile (16..256, at most the batch's own; 0 = planned) and the pair
 * count (0 = planned) of every later launch; used by tuning sweeps. */
int kvb_gemm_sk_set_plan(int mt, int pairs);

/* Process-wide tuning of kvb_gemm_bf16 / kvb_gemm_silu_bf16 (no reference
 * counterpart): the producer asks L2 for the weight K-steps `ksteps` ahead of
 * its TMA loads (cp.async.bulk.prefetch.tensor; 0 = off, the default; at most
 * 64). Applies to launches made after the call. */
int kvb_gemm_set_l2_prefetch(int ksteps);

/* ---------------------------------------- tensor-parallel all-reduce (NVLink) */

/* Size in bytes of the CUDA IPC handle kvb_comm_create writes. */
int kvb_comm_ipc_handle_size(void);

/* Per-rank communicator of a TP group (one process per GPU, current device).
 * Allocates this rank's symmetric area (flags, three partial-sum buffers of
 * max_bytes each, a result area) and writes its CUDA IPC handle to ipc_handle.
 * The caller gathers every rank's handle (rank order) over any channel and
 * passes them to kvb_comm_open_peers. Replaces the NCCL all-reduces of
 * linear.py:158-159 and embed_head.py:39-41 (NCCL stays for init/barriers). */
int kvb_comm_create(int rank, int world, size_t max_bytes, void** comm, void* ipc_handle);
int kvb_comm_open_peers(void* comm, const void* handles);
/* Device pointer of partial-sum buffer `index` (0..2): the row-parallel GEMM /
 * the embedding writes its rank-local [tokens, hidden] bf16 result there. */
int kvb_comm_data_buffer(void* comm, int index, void** ptr, size_t* bytes);
int kvb_comm_destroy(void* comm);

/* Alternative to kvb_comm_create/open_peers: attach to a symmetric area the
 * caller allocated and mapped on every rank (e.g. torch symmetric memory),
 * at least kvb_comm_area_size(max_bytes) bytes, zero-filled on every rank
 * before the first call. peer_bases[p] = rank p's area as mapped in this
 * process (256-byte aligned); multicast_base = the area's NVLink multicast
 * (NVLS) mapping, or 0 when the system has none. The area stays owned by the
 * caller; kvb_comm_destroy frees only the library's own counters. */
int kvb_comm_area_size(size_t max_bytes, size_t* bytes);
int kvb_comm_attach(int rank, int world, const uint64_t* peer_bases, uint64_t multicast_base, size_t area_bytes,
                    size_t max_bytes, void** comm);
/* Largest grid (blocks) of this communicator's kvb_allreduce_add_rmsnorm
 * launches, 1..256 (default 256; a block then handles several rows). Every
 * rank of the group must set the same value. Each block of a call spins,
 * holding its SM slot, until the same block has arrived on every peer: a
 * caller that runs two groups' calls concurrently on two streams caps both,
 * so that the two grids together leave SMs free for the kernels the peers
 * wait behind.
 * No reference counterpart (the reference issues one NCCL all-reduce at a
 * time, linear.py:158-159). */
int kvb_comm_set_max_blocks(void* comm, int max_blocks);
/* 1 when the communicator has a multicast mapping (switch-reduced modes). */
int kvb_comm_has_multicast(void* comm);
/* The exchange kvb_allreduce_add_rmsnorm runs for these arguments (host
 * only, no device work): plan[0] = 1 for the peer two-shot, plan[1] = 0 (peer
 * modes), 1 (switch one-shot) or 2 (switch two-shot). */
int kvb_allreduce_plan(int world, int has_multicast, int tokens, int hidden, int mode, int* plan);
/* This rank's result rows of the switch two-shot mode: passing them (from row
 * 0) as out / residual_out of kvb_allreduce_add_rmsnorm lets the kernel leave
 * the reduced rows where the switch delivered them instead of copying them
 * out; they stay valid until the next all-reduce call of the group. */
int kvb_comm_result_rows(void* comm, void** out_rows, void** residual_rows);

/* Fused all-reduce + residual add + RMSNorm over the TP group
 * (linear.py:156-160 followed by layernorm.py:114-140; with residual_in =
 * NULL the embedding all-reduce followed by qwen3.py:155-156):
 *   y = bf16(sum over ranks of buffer[data_index]) (fp32 sum in rank order),
 *   r = fp32(y) + fp32(residual_in) (or y), residual_out <- bf16(r),
 *   out = bf16(bf16(r * rsqrt(mean(r^2) + eps)) * weight).
 * Every rank of the group must make the same calls in the same order. mode:
 * 0 automatic, 1 one-shot (every rank reduces every row from the peers'
 * buffers), 2 two-shot (each rank reduces 1/N of the rows, then exchanges
 * results), 3 one-shot through the NVLink switch (multimem.ld_reduce, fp32
 * accumulation), 4 two-shot through the switch (reduce 1/N of the rows, then
 * multimem.st them to every rank); 3 and 4 need a multicast mapping
 * (kvb_comm_attach). Peer waits are
 * bounded (~1 s); on expiry the kernel raises device error bit 16 and returns.
 * residual_out may alias residual_in. Consecutive calls must use different
 * data buffers. */
int kvb_allreduce_add_rmsnorm(void* comm, int data_index, const void* residual_in, void* residual_out, void* out,
                              const void* weight, int tokens, int hidden, float eps, int mode, void* stream);

/* ------------------------------------------------------------------ sampler */

/* Sampler (sampler.py:7-66): token[b] = argmax_v(logits[b, v] / T[b] + g(b, v))
 * with Gumbel noise g = -log(-log(u)) from Philox4x32-10 keyed by *seed
 * (device int32), counter (b*vocab + v)/4, u = (top 23 bits + 0.5) / 2^23;
 * T[b] == 0 is greedy argmax. Ties pick the lowest index. Columns whose
 * logit/T cannot reach the bound set by the largest logit skip the noise
 * (exact: the noise is bounded by 24 ln 2).
 * logits bf16 [batch, vocab] with row stride; out int64 [batch]. The seed is
 * read, not advanced (the caller advances it, as sampler.py:59 does). */
int kvb_sample(const void* logits, int64_t row_stride, const float* temperatures, const int32_t* seed,
               int64_t* out, int batch, int vocab, void* stream);

/* Vocab-sharded sampler for ParallelLMHead (embed_head.py:56-66): the same
 * score over this rank's columns [vocab_offset, vocab_offset + shard_vocab)
 * of a vocab_total-wide row, written as (best score, global index) pairs to
 * best_val[b] / best_idx[b]. kvb_sample_combine then reduces world_size such
 * pairs per row (gathered as [world_size, batch]) to the token ids. The result
 * is identical to kvb_sample on the concatenated logits. */
int kvb_sample_partial(const void* logits, int64_t row_stride, const float* temperatures, const int32_t* seed,
                       float* best_val, int64_t* best_idx, int batch, int shard_vocab, int64_t vocab_offset,
                       int64_t vocab_total, void* stream);
int kvb_sample_combine(const float* vals, const int64_t* idxs, int world_size, int64_t* out, int batch,
                       void* stream);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* KAVOR_B200_H */
