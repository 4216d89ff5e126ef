// Shared device/host helpers for the ferrite B200 kernels (sm_100a only).
//
// Host side: status/error plumbing for the C ABI (thread-local last-error string,
// per-device SM count cache, optional host-side fault injection).
// Device side: vector load/store helpers, dtype conversion, bounded mbarrier
// waits, TMA (cp.async.bulk.tensor) issue, and tcgen05 / TMEM wrappers written
// from the PTX ISA description of those instructions.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>

#include "../../include/ferrite_b200.h"

namespace ferrite {

// --------------------------------------------------------------------------
// host: status + errors
// --------------------------------------------------------------------------

void set_error(const char* fmt, ...);
int fail(int code, const char* fmt, ...);
int num_sms(int device);
int current_device();
// Returns FERRITE_INJECTED_FAULT when the FERRITE_FAULT_INJECT environment
// variable names `op` (comma separated list, or "all"); 0 otherwise.
int injected_fault(const char* op);
// Checks cudaGetLastError() after a launch.
int check_launch(const char* what);

// Kernel launch with programmatic dependent launch (PDL) allowed: the kernel may
// be scheduled while the previous kernel in the stream is still finishing (its
// CTAs run their set-up, then wait in pdl_wait() until that kernel has completed
// and its memory is visible).  Hides the launch gap and the ramp-up between the
// back-to-back kernels of a step.  FERRITE_PDL=0 launches plainly.  Returns the
// launch's cudaError_t.
cudaError_t launch_k(const void* func, dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                     void** args);

// The same with thread-block clusters of `cluster_x` CTAs along x (the grid's x a
// multiple of it).
cudaError_t launch_k_cluster(const void* func, dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                             void** args, unsigned cluster_x);
// Clusters of `cluster_x` CTAs of `func` that fit on the device at once (0 on error).
int max_active_clusters(const void* func, dim3 block, size_t smem, unsigned cluster_x);

template <typename... KP>
inline cudaError_t launch_cluster_impl(void (*kern)(KP...), dim3 grid, dim3 block, size_t smem,
                                       cudaStream_t s, unsigned cluster_x, KP... v) {
  void* ptrs[sizeof...(KP) > 0 ? sizeof...(KP) : 1] = {(void*)&v...};
  return launch_k_cluster((const void*)kern, grid, block, smem, s, ptrs, cluster_x);
}
template <typename... KP, typename... A>
inline cudaError_t launch_pdl_cluster(void (*kern)(KP...), dim3 grid, dim3 block, size_t smem,
                                      cudaStream_t s, unsigned cluster_x, A&&... a) {
  return launch_cluster_impl<KP...>(kern, grid, block, smem, s, cluster_x, static_cast<KP>(a)...);
}

template <typename... KP>
inline cudaError_t launch_pdl_impl(void (*kern)(KP...), dim3 grid, dim3 block, size_t smem,
                                   cudaStream_t s, KP... v) {
  void* ptrs[sizeof...(KP) > 0 ? sizeof...(KP) : 1] = {(void*)&v...};
  return launch_k((const void*)kern, grid, block, smem, s, ptrs);
}
// launch_pdl(kernel, grid, block, smem, stream, args...): arguments converted to
// the kernel's parameter types.
template <typename... KP, typename... A>
inline cudaError_t launch_pdl(void (*kern)(KP...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t s, A&&... a) {
  return launch_pdl_impl<KP...>(kern, grid, block, smem, s, static_cast<KP>(a)...);
}
// Encodes a 2-D tiled TMA descriptor (inner dimension first) with 128-byte
// swizzle; returns 0 or a FERRITE_* code with the error set.
int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
                 int elem_bytes, uint64_t inner, uint64_t outer,
                 uint64_t row_stride_bytes, uint32_t box_inner,
                 uint32_t box_outer, CUtensorMapSwizzle swizzle);
// Same for a 3-D tensor (inner, middle, outer).
int make_tmap_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
                 int elem_bytes, uint64_t d0, uint64_t d1, uint64_t d2,
                 uint64_t stride1_bytes, uint64_t stride2_bytes,
                 uint32_t box0, uint32_t box1, uint32_t box2,
                 CUtensorMapSwizzle swizzle);
// 4-D map (dims d0 innermost .. d3, byte strides of dims 1..3).
int make_tmap_4d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
                 int elem_bytes, const uint64_t dims[4], const uint64_t strides_bytes[3],
                 const uint32_t box[4], CUtensorMapSwizzle swizzle);

// Device status word, one per translation unit and device (internal linkage,
// so the translation units need no relocatable device code).  Set by bounded
// waits that expire.  Each translation unit that waits exports a reader that
// ferrite_device_status() polls.
static __device__ int g_device_status = 0;
// Reads (and optionally clears) this translation unit's status word; the
// stream must already be synchronised.
#define FERRITE_DEFINE_STATUS_READER(NAME)                                  \
  int NAME(int clear) {                                                     \
    int v = 0;                                                              \
    if (cudaMemcpyFromSymbol(&v, g_device_status, sizeof(int)) != cudaSuccess) \
      return FERRITE_LAUNCH_FAILED;                                         \
    if (clear && v != 0) {                                                  \
      int zero = 0;                                                         \
      cudaMemcpyToSymbol(g_device_status, &zero, sizeof(int));              \
    }                                                                       \
    return v;                                                               \
  }
int status_gemm(int clear);
int status_attention(int clear);
int status_rmsnorm(int clear);

// --------------------------------------------------------------------------
// device: dtype helpers
// --------------------------------------------------------------------------

template <typename T>
struct DT;
template <>
struct DT<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
};
template <>
struct DT<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) {
    return __bfloat162float(v);
  }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) {
    return __float2bfloat16_rn(v);
  }
};
template <>
struct DT<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) {
    return __float2half_rn(v);
  }
};

// Streaming 16-byte global load that does not allocate in L1.
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
// Ordinary cached 16-byte read-only load (used for small reused vectors such as
// the norm weight).
__device__ __forceinline__ uint4 ld_v4(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}
__device__ __forceinline__ void st_v4(void* p, uint4 v) {
  *reinterpret_cast<uint4*>(p) = v;
}
// Streaming 16-byte store (evict-first).
__device__ __forceinline__ void st_stream_v4(void* p, uint4 v) {
  __stcs(reinterpret_cast<uint4*>(p), v);
}

// Programmatic dependent launch, device side.  pdl_launch_dependents(): this CTA
// lets the next kernel in the stream be scheduled (it runs once every CTA of this
// grid has started or exited).  pdl_wait(): block until the previous kernel in the
// stream has completed and its writes are visible; every thread calls it before
// its first global-memory access.  Both are no-ops for a plain launch.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Upper bound on any single device-side wait (nanoseconds of %globaltimer).
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ void report_timeout(int where) {
  atomicCAS(&g_device_status, 0, FERRITE_DEVICE_TIMEOUT);
  (void)where;
}

// --------------------------------------------------------------------------
// device: shared-memory addressing, mbarriers
// --------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar,
                                                      uint32_t bytes) {
  asm volatile(
      "mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for phase `parity` of `bar`, at most `limit_ns` of %globaltimer.
// Returns false (and records FERRITE_DEVICE_TIMEOUT in the device status word)
// if the wait expired or if *abort became non-zero while waiting; callers then
// skip their remaining work and fall through to the CTA's teardown.
__device__ __forceinline__ bool mbar_wait_ns(uint64_t* bar, uint32_t parity,
                                             volatile int* abort, int where,
                                             uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++spins & 255u) == 0) {
      if (*abort) return false;
      if (globaltimer_ns() - t0 > limit_ns) {
        report_timeout(where);
        *abort = 1;
        return false;
      }
    }
  }
}
// The kernels' wait: the same, with the library-wide limit kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          volatile int* abort, int where) {
  return mbar_wait_ns(bar, parity, abort, where, kWaitLimitNs);
}

// --------------------------------------------------------------------------
// device: TMA (tiled bulk tensor copies, no multicast)
// --------------------------------------------------------------------------

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map,
                                            uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::"
      "bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map,
                                            uint64_t* bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::"
      "bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map,
                                            uint64_t* bar, int c0, int c1, int c2,
                                            int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::"
      "bytes [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// Prefetch of a 4-D box into L2 (no shared-memory destination, no completion).
__device__ __forceinline__ void tma_prefetch_4d(const CUtensorMap* map, int c0, int c1, int c2, int c3) {
  asm volatile("cp.async.bulk.prefetch.tensor.4d.L2.global.tile [%0, {%1, %2, %3, %4}];" ::"l"(map), "r"(c0),
               "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}

// L2 cache policies for the .L2::cache_hint forms below: evict_last keeps lines
// resident ahead of normal traffic (scratch that is read back soon), evict_first
// lets them go first (data read for the last time).
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void tma_load_4d_hint(void* dst, const CUtensorMap* map, uint64_t* bar, int c0,
                                                 int c1, int c2, int c3, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5, %6}], [%2], %7;" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void tma_store_4d_hint(const CUtensorMap* map, const void* src, int c0, int c1,
                                                  int c2, int c3, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%2, %3, %4, %5}], [%1], %6;" ::"l"(map),
      "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "l"(policy)
      : "memory");
}

// TMA tiled store shared -> global (bulk-group completion; no multicast).
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int c0,
                                             int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(map),
      "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int c0,
                                             int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(map),
      "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int c0,
                                             int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(map),
      "r"(smem_u32(src)), "r"(c0), "r"(c1)
      : "memory");
}
// Wait until at most one of this thread's committed bulk groups still reads shared memory.
__device__ __forceinline__ void bulk_wait_group_read1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait until the bulk groups this thread committed have finished READING shared memory.
__device__ __forceinline__ void bulk_wait_group_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Wait until the bulk groups this thread committed have completed.
__device__ __forceinline__ void bulk_wait_group0() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
// Wait until all but the most recent of this thread's bulk groups have completed.
__device__ __forceinline__ void bulk_wait_group1() {
  asm volatile("cp.async.bulk.wait_group 1;" ::: "memory");
}

// --------------------------------------------------------------------------
// device: inter-CTA signalling in global memory (gpu scope)
// --------------------------------------------------------------------------

// Orders this thread's async-proxy (TMA) global accesses with its generic-proxy
// ones: after a completed TMA store and before a release that publishes it, and
// after an acquire and before TMA loads of what it published.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int ld_relaxed_gpu(const int* p) {
  int v;
  asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(int* p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_gpu(int* p, int v) {
  asm volatile("st.relaxed.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// atomic add with acquire-release semantics at gpu scope; returns the old value
__device__ __forceinline__ int atom_add_acq_rel_gpu(int* p, int v) {
  int old;
  asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ int atom_cas_gpu(int* p, int cmp, int v) {
  int old;
  asm volatile("atom.cas.relaxed.gpu.global.b32 %0, [%1], %2, %3;" : "=r"(old) : "l"(p), "r"(cmp), "r"(v) : "memory");
  return old;
}
// Release store / acquire load of a shared-memory word at CTA scope.
__device__ __forceinline__ void st_release_cta_shared(int* p, int v) {
  asm volatile("st.release.cta.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_cta_shared(const int* p) {
  int v;
  asm volatile("ld.acquire.cta.shared::cta.b32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
  return v;
}
__device__ __forceinline__ void red_add_release_gpu(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Drops the 128-byte L2 line at `p` without writing it back (its contents become
// undefined): for scratch that has been read for the last time.
__device__ __forceinline__ void discard_l2_line(const void* p) {
  asm volatile("discard.global.L2 [%0], 128;" ::"l"(p) : "memory");
}
__device__ __forceinline__ void mbar_inval(uint64_t* bar) {
  asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Untiled bulk copy global -> shared (no multicast): `bytes` must be a multiple
// of 16 and both addresses 16-byte aligned; completes `bytes` transactions on bar.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, "
      "[%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Named barrier over `count` threads (a multiple of 32), id 1..15.
__device__ __forceinline__ void named_barrier(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// --------------------------------------------------------------------------
// device: tcgen05 / TMEM
// --------------------------------------------------------------------------

// Allocate `ncols` TMEM columns (power of two >= 32); the base address is written
// to shared memory at `dst`.  Must be executed by one full warp.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile(
      "tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
          smem_u32(dst)),
      "r"(ncols)
      : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::
                   : "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(
                   taddr),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Arrive (once) on `bar` when all previously issued tcgen05.mma of this thread
// have completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
      "[%0];" ::"r"(smem_u32(bar))
      : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16 (bf16/f16 in, f32 acc).
__device__ __forceinline__ void tc_mma_f16_ss(uint32_t d_tmem, uint64_t adesc,
                                              uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(
          d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc], kind::f16.  A is read from TMEM
// (M lanes x K/2 columns of packed 16-bit pairs).
__device__ __forceinline__ void tc_mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem,
                                              uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(
          d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Load 32 consecutive f32 columns of this thread's TMEM lane.
// Shape 32x32b: warp w (w = warp id % 4) may only address lanes 32w..32w+31;
// thread t of the warp receives lane 32w+t.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, "
      "[%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
        "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]),
        "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
        "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]),
        "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// Store 32 consecutive 32-bit columns into this thread's TMEM lane.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]),
      "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]),
      "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]),
      "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
// 2^x with the hardware approximation (ex2.approx.ftz.f32: relative error
// ~2^-22, subnormal results flushed to zero).  Used for softmax numerators that
// are rounded to bf16/f16 afterwards.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// Store 8 consecutive 32-bit columns into this thread's TMEM lane.
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
      : "memory");
}
// Store 16 consecutive 32-bit columns into this thread's TMEM lane.
__device__ __forceinline__ void tmem_st16(uint32_t taddr,
                                          const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]),
      "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]),
      "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// Shared-memory matrix descriptor for tcgen05.mma (sm_100 "version 1" format):
//   bits  0-13  start address >> 4
//   bits 16-29  leading-dimension byte offset >> 4
//   bits 32-45  stride-dimension byte offset >> 4
//   bits 46-47  version (1)
//   bits 49-51  base offset (0: every swizzle atom here is 1024-byte aligned)
//   bit  52     LBO mode (0)
//   bits 61-63  layout: 0 none, 2 = 128-byte swizzle, 4 = 64B, 6 = 32B
// For 128-byte swizzled tiles:
//   K-major  (rows of 64 bf16 = 128 B, 8-row atoms of 1 KiB):
//            SBO = 1024 (next 8 rows), LBO unused (1); a K step of 16 elements
//            advances the start address by 32 bytes inside the atom.
//   MN-major (rows of 64 MN-contiguous elements per k, 8-k atoms of 1 KiB):
//            LBO = byte distance between 64-element MN chunks,
//            SBO = 1024 (next 8 k); a K step of 16 advances by 2048 bytes.
__device__ __forceinline__ uint64_t make_sdesc(uint32_t saddr, uint32_t lbo,
                                               uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // version
  d |= (uint64_t)2 << 61;  // 128-byte swizzle
  return d;
}

// Descriptor of the same layout `byte_off` bytes further into shared memory.
// The start-address field holds addr >> 4 in 14 bits; shared-memory addresses
// stay below 2^18 bytes, so adding (byte_off >> 4) never carries out of it.
// Lets issuing code build a descriptor once and add compile-time offsets per MMA.
__device__ __forceinline__ uint64_t sdesc_at(uint64_t desc, uint32_t byte_off) {
  return desc + (uint64_t)(byte_off >> 4);
}

// Instruction descriptor for kind::f16 with f32 accumulation.
//   bits 4-5 D format (1 = f32), 7-9 A format, 10-12 B format (0 f16, 1 bf16),
//   bit 15 A major (0 K, 1 MN), bit 16 B major, bits 17-22 N>>3, 24-28 M>>4.
__host__ __device__ constexpr uint32_t make_idesc_f16(int M, int N, bool bf16,
                                                      bool a_mn, bool b_mn) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) |
         ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ uint32_t elect_one_sync() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .b32 rx;\n\t.reg .pred px;\n\t"
      "elect.sync rx|px, %1;\n\t"
      "selp.b32 %0, 1, 0, px;\n\t}"
      : "=r"(pred)
      : "r"(0xffffffffu));
  return pred;
}

// --------------------------------------------------------------------------
// device: CTA pairs (cluster of 2) for tcgen05 cta_group::2
// --------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the variable at local shared address `p` in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(const void* p, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(smem_u32(p)), "r"(rank));
  return d;
}
// All threads of every CTA of the cluster.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive on an mbarrier of another CTA of the cluster (address from mapa_shared).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster_addr) : "memory");
}
// TMEM allocation shared by the CTA pair: one warp of each CTA (the same warp index)
// executes it with the same destination offset; both CTAs get the same columns.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D (M = 256 over the pair: rows 0-127 in the leader's TMEM, 128-255 in the peer's)
// (+)= A * B, issued by one thread of the leader (even rank).  The descriptors give
// this CTA's shared-memory offsets; the peer's operand halves sit at the same offsets.
__device__ __forceinline__ void tc_mma_pair_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once, on the mbarrier at local offset `bar` of every CTA in `cta_mask`, when the
// pair MMAs issued so far by this thread have completed.
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}
// 2-D TMA load into this CTA's shared memory whose completion is counted on an
// mbarrier of the pair's leader (`bar_cluster_addr` from mapa_shared).  No multicast:
// each CTA loads only its own operand half.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster_addr,
                                                 int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(bar_cluster_addr), "r"(c0), "r"(c1)
      : "memory");
}

// Per-warpgroup register re-allocation (all 128 threads of a warpgroup execute
// it).  A kernel that uses it must release at least as many registers (dec) as
// it acquires (inc), counted against its launch allocation.
template <int N>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// --------------------------------------------------------------------------
// device: packed f32 pairs (sm_100 FFMA2 / FADD2 / FMUL2: two IEEE f32
// operations per instruction, each rounded exactly like its scalar form)
// --------------------------------------------------------------------------
__device__ __forceinline__ uint64_t f2_make(float lo, float hi) {
  uint64_t d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(lo), "f"(hi));
  return d;
}
__device__ __forceinline__ uint64_t f2_make_bits(uint32_t lo, uint32_t hi) {
  uint64_t d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "r"(lo), "r"(hi));
  return d;
}
__device__ __forceinline__ float f2_lo(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float f2_hi(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// max of three f32 (one instruction on sm_100)
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

}  // namespace ferrite
