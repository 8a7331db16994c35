// Shared device/host helpers for the kavor_b200 kernels (sm_100a only).
//
// Error convention of every extern "C" entry point (include/kavor_b200.h):
//   0  = success
//   <0 = invalid argument, detected on the host before any launch
//   >0 = a cudaError_t returned by the launch
// A human-readable message for the last failure on the calling host thread is
// kept in a thread-local buffer (kvb_last_error()).
//
// Device-side failures (an index that would leave its buffer, an mbarrier wait
// that ran out of its iteration budget) never trap: the kernel ORs a bit into a
// per-translation-unit __device__ error word, skips the access or returns, and
// the host reads the words back with kvb_device_error().
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stddef.h>

namespace kvb {

using bf16 = __nv_bfloat16;

enum Status : int {
  kOk = 0,
  kInvalid = -1,       // bad pointer, size or stride
  kUnsupported = -2,   // shape outside what the kernels are built for
  kWorkspace = -3,     // caller-provided workspace too small
  kNoEncoder = -4,     // cuTensorMapEncodeTiled could not be resolved
  kEncode = -5,        // cuTensorMapEncodeTiled rejected the tensor map
};

// Device error bits (ORed into the per-TU error word).
enum DeviceError : unsigned {
  kErrBlockTable = 1u << 0,   // block id out of [0, num_blocks) or table column out of range
  kErrSlot = 1u << 1,         // slot_mapping entry outside the cache
  kErrTimeout = 1u << 2,      // bounded mbarrier / flag wait gave up
  kErrTokenId = 1u << 3,      // embedding id outside the vocabulary
  kErrPeerTimeout = 1u << 4,  // cross-GPU flag wait gave up
  kErrConfig = 1u << 5,       // a launch configuration the kernel cannot serve (work skipped)
};

// Host-side error message helpers (defined in capi.cu).
int set_error(int status, const char* fmt, ...);
int cuda_status(cudaError_t e, const char* where);

// cuTensorMapEncodeTiled, resolved once through the runtime's driver entry
// point (the library links no libcuda); NULL when the driver lacks it.
inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
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

// SM count of the current device, cached per device (148, the B200's, when it
// cannot be read: host-only planning on a machine without a GPU).
inline int device_sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return 148;
  }
  if (!cached[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) cudaGetLastError();
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

// Spin budget for every device-side wait: ~2^31 SM cycles (about a second at
// 1.9 GHz). Waits that exceed it set kErrTimeout and give up.
constexpr long long kSpinCycles = 1ll << 31;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(bar),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false (and sets kErrTimeout in *err) when the phase
// did not complete within kSpinCycles.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, unsigned* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kSpinCycles) {
      atomicOr(err, (unsigned)kErrTimeout);
      return false;
    }
  }
  return true;
}

// ---------------------------------------------------------------- TMA
// 4-D tiled bulk tensor load into shared memory, completion on an mbarrier.
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            int c3, uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------- cp.async
__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;  // src-size 0 zero-fills the 16 bytes
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ---------------------------------------------------------------- warp MMA
__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                            uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                                  uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// D = A(16x16 bf16, row) * B(16x8 bf16, col) + D, fp32 accumulate.
__device__ __forceinline__ void mma_bf16_16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Named barrier over a subset of warps (id 0 is __syncthreads).
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---------------------------------------------------- programmatic dependent launch
// Every kernel calls kernel_entry() before its first access to memory that
// another kernel writes (at its start, or after its set-up): wait until the grids it depends on
// have completed and their writes are visible (griddepcontrol.wait; returns at
// once when the kernel was launched without a programmatic dependency). With
// programmatic launch on (kvb_set_pdl), it then lets the next kernel of the
// stream be scheduled early (it stops at its own wait), so that kernel's launch
// and CTA dispatch overlap this kernel's run; off (the default), the next
// kernel starts after this one ends, as with plain launches. Nothing that a
// kernel before it writes is read, and nothing is written, before the wait
// (the GEMM requests its first weight tiles, which no kernel writes, before
// it). The switch is a per-translation-unit constant, written by kvb_set_pdl
// through set_pdl_trigger_<tag>().
static __constant__ int c_pdl_trigger = 0;

__device__ __forceinline__ void kernel_entry() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (c_pdl_trigger) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Launches made with programmatic stream serialization (kvb_set_pdl) or as
// plain stream-ordered launches (the default).
bool pdl_enabled();

template <typename... Params, typename... Args>
cudaError_t launch_kernel(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                          Args&&... args) {
  if (!pdl_enabled()) {
    kernel<<<grid, block, smem, stream>>>(static_cast<Args&&>(args)...);
    return cudaGetLastError();
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

}  // namespace kvb

// Every translation unit that launches kernels defines its own error word and
// a host reader; capi.cu ORs them together for kvb_device_error(). It also
// defines the setter of its programmatic-launch switch (kvb_set_pdl).
#define KVB_DEFINE_ERROR_WORD(tag)                                                  \
  namespace kvb {                                                                   \
  __device__ unsigned g_err_##tag = 0;                                              \
  int read_device_error_##tag(unsigned* out, int clear) {                           \
    cudaError_t e = cudaMemcpyFromSymbol(out, g_err_##tag, sizeof(unsigned));       \
    if (e != cudaSuccess) return cuda_status(e, "read device error word");          \
    if (clear) {                                                                    \
      unsigned z = 0;                                                               \
      e = cudaMemcpyToSymbol(g_err_##tag, &z, sizeof(unsigned));                    \
      if (e != cudaSuccess) return cuda_status(e, "clear device error word");       \
    }                                                                               \
    return 0;                                                                       \
  }                                                                                 \
  int set_pdl_trigger_##tag(int on) {                                               \
    cudaError_t e = cudaMemcpyToSymbol(c_pdl_trigger, &on, sizeof(int));            \
    return e == cudaSuccess ? 0 : cuda_status(e, "set launch mode");                \
  }                                                                                 \
  }
