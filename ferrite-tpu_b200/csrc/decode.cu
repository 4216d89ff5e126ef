// Decode attention: one new query row per (batch, head) against a static KV cache --
// the serving engine's decode step of the reference (src/ferrite/serving/engine.py:
// _write_cache :98-104 stores the new token's K/V row at pos[b], then
// _cache_attention :89-95 takes softmax(scale * q K^T) V with every cache position
// after pos[b] masked to -1e30).
//
// HBM-bound: every cache row up to pos[b] is read once (its K and V), nothing else
// of size.  A masked position's softmax weight is exp(-1e30 - max) = 0 exactly in
// f32, so positions after pos[b] are not read at all.
//
// Work layout: one thread-block cluster of C CTAs (C = 1..8, chosen on the host so
// that the grid covers the SMs about twice) per (batch, head) slice.  The rows
// [0, pos] are split evenly over the cluster's CTAs on the device (pos is only known
// there).  A row of d elements is read by d / EPV lanes, 16 bytes each (EPV = 8
// elements for bf16/f16, 4 for f32), so a warp reads 32 / (d / EPV) rows at once.
// Each such lane group keeps an online-softmax state (running max, sum, f32
// accumulator) over its rows, kUnroll rows per step, staged through a per-thread
// shared-memory ring of cp.async copies kStages - 1 steps ahead.  The groups are merged in shared memory;
// rank 0 of the cluster then merges the CTAs' states through distributed shared
// memory and writes the output row: no global scratch and no second kernel.
//
// The cache write is fused: row pos[b] is read from k_new / v_new (never from the
// cache), and the one CTA whose rows include pos[b] stores that row into the cache,
// so no CTA reads a cache row that this launch writes.
#include <cooperative_groups.h>

#include <atomic>
#include <cmath>
#include <cstdlib>
#include <type_traits>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace ferrite {
namespace decode {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kUnroll = 4;
constexpr int kStages = 3;
// K/V staging ring per CTA: kStages batches x kUnroll rows x (K, V) x 16 bytes per thread.
constexpr int kRingBytes = kStages * kUnroll * 2 * kThreads * 16;
constexpr int kMaxCluster = 8;
constexpr int kPrefetchBytes = 32 * 1024;  // per CTA, of K and of V, ahead of the launch wait
constexpr float kLog2e = 1.4426950408889634f;

// 16-byte global -> shared asynchronous copy (cached in L2 only), and its group
// commit / wait; wait_group N returns once at most N of this thread's groups are pending.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// 16 bytes of T -> EPV floats.
template <typename T>
__device__ __forceinline__ void unpack(const uint4& u, float (&f)[16 / sizeof(T)]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
  if constexpr (std::is_same_v<T, float>) {
#pragma unroll
    for (int i = 0; i < 4; ++i) f[i] = __uint_as_float(w[i]);
  } else if constexpr (std::is_same_v<T, __nv_bfloat16>) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {  // bf16 -> f32 is exact: the bits move up 16 places
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 p = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      f[2 * i] = p.x;
      f[2 * i + 1] = p.y;
    }
  }
}

// Grid (b * h, C), cluster (1, C, 1), kThreads threads.  q, k_new, v_new: row
// (b, h) at b * ld_new + h * D; caches [b, h, max_len, D]; out [b, h, D].
template <int D, typename T>
__global__ void __launch_bounds__(kThreads, 2)
    decode_attn_kernel(const T* __restrict__ q, const T* __restrict__ k_new,
                       const T* __restrict__ v_new, T* __restrict__ k_cache,
                       T* __restrict__ v_cache, const int64_t* __restrict__ pos,
                       T* __restrict__ out, int h, int64_t max_len, int64_t ld_new, float qscale) {
  constexpr int EPV = 16 / (int)sizeof(T);  // elements per 16-byte lane vector
  constexpr int LPR = D / EPV;              // lanes per row
  constexpr int RPW = 32 / LPR;             // rows per warp step
  constexpr int G = kWarps * RPW;           // lane groups per CTA
  static_assert(LPR >= 1 && LPR <= 32 && (LPR & (LPR - 1)) == 0, "row must map to a power-of-two lane group");
  __shared__ __align__(16) float s_acc[G][D];
  __shared__ float s_m[G], s_l[G];
  __shared__ __align__(16) float c_acc[D];
  __shared__ float c_ml[2];

  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int csize = (int)cluster.num_blocks();
  const int64_t slice = blockIdx.x;
  const int64_t bi = slice / h, hi = slice % h;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane % LPR;      // which 16 bytes of the row this lane reads
  const int row_in_warp = lane / LPR;
  const int grp = warp * RPW + row_in_warp;

  pdl_launch_dependents();
  // Pull the first of this CTA's cache rows into L2 while the previous kernel finishes
  // (a launch that follows through programmatic dependent launch starts early): up to
  // kPrefetchBytes of K and of V, what its first copies ask for.  Prefetching the whole
  // range was slower at a full cache (it competes with the previous launch's traffic);
  // this cap measured best.  pos may still be in flight from an earlier kernel of the
  // stream, so this read (relaxed) only steers a prefetch, which returns no data; the
  // rows themselves are read after pdl_wait().
  if ((int)threadIdx.x < 2) {
    int64_t p0;
    asm volatile("ld.relaxed.gpu.global.s64 %0, [%1];" : "=l"(p0) : "l"(pos + bi) : "memory");
    if (p0 >= 0 && p0 < max_len) {
      const int64_t n0 = p0 + 1, chunk0 = (n0 + csize - 1) / csize;
      const int64_t b0 = min((int64_t)rank * chunk0, n0), e0 = min(b0 + chunk0, n0);
      if (e0 > b0) {
        const T* base = (threadIdx.x == 0 ? k_cache : v_cache) + (slice * max_len + b0) * D;
        const int64_t bytes = min((e0 - b0) * D * (int64_t)sizeof(T), (int64_t)kPrefetchBytes);  // a multiple of 16
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(base), "r"((uint32_t)bytes) : "memory");
      }
    }
  }
  pdl_wait();  // the previous kernel in the stream has finished (it may have written q or the cache)
  float qf[EPV], acc[EPV];
  unpack<T>(ld_v4(q + bi * ld_new + hi * D + sub * EPV), qf);
#pragma unroll
  for (int e = 0; e < EPV; ++e) {
    qf[e] *= qscale;  // scores come out in log2 units: exp(s - m) = 2^(s' - m')
    acc[e] = 0.f;
  }

  const int64_t p = pos[bi];
  const bool valid = p >= 0 && p < max_len;
  // rows [begin, end) of [0, p] for this CTA (empty when pos is invalid)
  const int64_t n = valid ? p + 1 : 0;
  const int64_t chunk = (n + csize - 1) / csize;
  const int64_t begin = min((int64_t)rank * chunk, n);
  const int64_t end = min(begin + chunk, n);

  const T* knew = k_new ? k_new + bi * ld_new + hi * D : nullptr;
  const T* vnew = v_new ? v_new + bi * ld_new + hi * D : nullptr;
  T* kc = k_cache + slice * max_len * D;
  T* vc = v_cache + slice * max_len * D;

  if (knew && p >= begin && p < end) {  // fused cache write of the new row
    if ((int)threadIdx.x < LPR)
      st_v4(kc + p * D + threadIdx.x * EPV, ld_v4(knew + threadIdx.x * EPV));
    else if ((int)threadIdx.x < 2 * LPR)
      st_v4(vc + p * D + (threadIdx.x - LPR) * EPV, ld_v4(vnew + (threadIdx.x - LPR) * EPV));
  }

  // Rows of lane group grp: begin + grp + k * G, k = 0, 1, ...; batch t holds k = t * kUnroll
  // .. t * kUnroll + kUnroll - 1.  Each lane stages its 16-byte pieces of a batch's K and V
  // rows in its own slots of a kStages-deep shared-memory ring with cp.async (16-byte,
  // L2 only), kStages - 1 batches ahead of the one it consumes: ~96 KB in flight per CTA
  // without holding registers.  A lane reads back only the bytes it copied itself, so
  // cp.async.wait_group (this thread's own copies) is the only wait.  The batch count is
  // warp-uniform (the shuffles below need the whole warp); rows past `end` are masked.
  extern __shared__ __align__(16) uint4 ring[];  // [kStages][kUnroll][K, V][kThreads]
  auto slot = [&](int st, int u, int kv) -> uint4* {
    return &ring[((st * kUnroll + u) * 2 + kv) * kThreads + threadIdx.x];
  };
  const int64_t step = (int64_t)kUnroll * G;
  const int64_t jw0 = begin + warp * RPW;
  const int64_t nb = jw0 < end ? (end - jw0 + step - 1) / step : 0;
  auto issue = [&](int64_t t) {
    const int st = (int)(t % kStages);
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t j = jw0 + t * step + row_in_warp + (int64_t)u * G;
      if (j < end) {
        const T* kr = (j == p && knew) ? knew : kc + j * D;
        const T* vr = (j == p && vnew) ? vnew : vc + j * D;
        cp_async16(slot(st, u, 0), kr + sub * EPV);
        cp_async16(slot(st, u, 1), vr + sub * EPV);
      }
    }
  };
#pragma unroll
  for (int t = 0; t < kStages - 1; ++t) {
    if (t < nb) issue(t);
    cp_async_commit();  // possibly empty: keeps the group count per batch fixed
  }
  float m = -INFINITY, l = 0.f;
  for (int64_t t = 0; t < nb; ++t) {
    if (t + kStages - 1 < nb) issue(t + kStages - 1);
    cp_async_commit();
    cp_async_wait<kStages - 1>();  // batch t's copies (this thread's) have landed
    const int st = (int)(t % kStages);
    const int64_t jw = jw0 + t * step;
    uint4 ka[kUnroll], va[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const bool in = jw + row_in_warp + (int64_t)u * G < end;
      ka[u] = in ? *slot(st, u, 0) : make_uint4(0u, 0u, 0u, 0u);
      va[u] = in ? *slot(st, u, 1) : make_uint4(0u, 0u, 0u, 0u);
    }
    float s[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      float kf[EPV];
      unpack<T>(ka[u], kf);
      float a = 0.f;
#pragma unroll
      for (int e = 0; e < EPV; ++e) a = fmaf(qf[e], kf[e], a);
      s[u] = a;
    }
#pragma unroll
    for (int off = LPR / 2; off > 0; off >>= 1)
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) s[u] += __shfl_xor_sync(0xffffffffu, s[u], off);
    float mx = m;
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t j = jw + row_in_warp + (int64_t)u * G;
      s[u] = j < end ? s[u] : -INFINITY;
      mx = fmaxf(mx, s[u]);
    }
    if (mx != -INFINITY) {  // uniform inside a lane group
      const float c = ex2_approx(m - mx);  // 0 while m is still -inf
      l *= c;
#pragma unroll
      for (int e = 0; e < EPV; ++e) acc[e] *= c;
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const float pu = ex2_approx(s[u] - mx);  // 0 for a masked row (whose v is zeros)
        float vf[EPV];
        unpack<T>(va[u], vf);
        l += pu;
#pragma unroll
        for (int e = 0; e < EPV; ++e) acc[e] = fmaf(pu, vf[e], acc[e]);
      }
      m = mx;
    }
  }
  cp_async_wait<0>();  // only empty groups can remain; nothing is in flight at exit

  // merge the lane groups of this CTA
#pragma unroll
  for (int e = 0; e < EPV; ++e) s_acc[grp][sub * EPV + e] = acc[e];
  if (sub == 0) {
    s_m[grp] = m;
    s_l[grp] = l;
  }
  __syncthreads();
  if ((int)threadIdx.x < D) {
    const int t = threadIdx.x;
    float M = -INFINITY;
#pragma unroll
    for (int g = 0; g < G; ++g) M = fmaxf(M, s_m[g]);
    float L = 0.f, A = 0.f;
    if (M != -INFINITY) {
#pragma unroll 8
      for (int g = 0; g < G; ++g) {
        const float w = ex2_approx(s_m[g] - M);
        L = fmaf(s_l[g], w, L);
        A = fmaf(s_acc[g][t], w, A);
      }
    }
    c_acc[t] = A;
    if (t == 0) {
      c_ml[0] = M;
      c_ml[1] = L;
    }
  }
  cluster.sync();  // every CTA's (max, sum, acc) is visible to the cluster

  if (rank == 0 && (int)threadIdx.x < D) {
    const int t = threadIdx.x;
    float M = -INFINITY;
    for (int r = 0; r < csize; ++r) M = fmaxf(M, cluster.map_shared_rank(c_ml, r)[0]);
    float L = 0.f, A = 0.f;
    if (M != -INFINITY) {
      for (int r = 0; r < csize; ++r) {
        const float* ml = cluster.map_shared_rank(c_ml, r);
        const float w = ex2_approx(ml[0] - M);
        L = fmaf(ml[1], w, L);
        A = fmaf(cluster.map_shared_rank(c_acc, r)[t], w, A);
      }
    }
    out[slice * D + t] = DT<T>::from_f(valid ? A / L : NAN);
  }
  cluster.sync();  // the other CTAs' shared memory stays alive until rank 0 has read it
}

// Cluster size for b*h slices of up to max_len rows: the largest C (up to 8) whose grid
// of b*h*C CTAs still fits in one wave (`slots` = SMs x resident CTAs per SM) while every
// CTA keeps at least one row per lane group of a full cache.  One wave matters more than
// more CTAs: a partial second wave repeats the whole per-CTA latency chain.
static int pick_cluster(int64_t bh, int64_t max_len, int groups, int64_t slots) {
  int c = 1;
  while (c < kMaxCluster && bh * 2 * c <= slots && max_len / (2 * c) >= groups) c *= 2;
  return c;
}

template <int D, typename T>
static int launch(cudaStream_t s, const void* q, const void* k_new, const void* v_new,
                  void* k_cache, void* v_cache, const int64_t* pos, void* out, int64_t b,
                  int64_t h, int64_t max_len, int64_t ld_new, float scale) {
  constexpr int EPV = 16 / (int)sizeof(T);
  constexpr int G = kWarps * (32 / (D / EPV));
  const int64_t bh = b * h;
  const int dev = current_device();
  // resident CTAs per SM of this instantiation, per device (set once; racing first calls
  // store the same value)
  static std::atomic<int> occ[64];
  if (dev < 0 || dev >= 64) return fail(FERRITE_LAUNCH_FAILED, "attn_decode: device ordinal %d", dev);
  if (occ[dev].load(std::memory_order_relaxed) == 0) {
    cudaError_t e = cudaFuncSetAttribute(decode_attn_kernel<D, T>, cudaFuncAttributeMaxDynamicSharedMemorySize, kRingBytes);
    if (e != cudaSuccess) return fail(FERRITE_LAUNCH_FAILED, "attn_decode: shared memory attribute: %s", cudaGetErrorString(e));
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_attn_kernel<D, T>, kThreads, kRingBytes) != cudaSuccess || n < 1) n = 1;
    occ[dev].store(n, std::memory_order_relaxed);
  }
  int c = pick_cluster(bh, max_len, G, (int64_t)num_sms(dev) * occ[dev].load(std::memory_order_relaxed));
  if (const char* e = std::getenv("FERRITE_DECODE_CLUSTER")) {  // A/B override: 1, 2, 4 or 8
    const int v = std::atoi(e);
    if (v == 1 || v == 2 || v == 4 || v == 8) c = v;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)bh, (unsigned)c, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kRingBytes;
  cfg.stream = s;
  // Programmatic dependent launch, as for the other kernels (FERRITE_PDL=0 turns it off):
  // the CTAs of the next launch in the stream are scheduled as this one's CTAs retire and
  // wait in griddepcontrol.wait, which hides the launch gap between per-layer calls.
  static const bool pdl = [] {
    const char* e = std::getenv("FERRITE_PDL");
    return !(e && *e && std::atoi(e) == 0);
  }();
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = (unsigned)c;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, decode_attn_kernel<D, T>, (const T*)q, (const T*)k_new,
                                     (const T*)v_new, (T*)k_cache, (T*)v_cache, pos, (T*)out, (int)h,
                                     max_len, ld_new, scale * kLog2e);
  if (e != cudaSuccess) return fail(FERRITE_LAUNCH_FAILED, "attn_decode: %s", cudaGetErrorString(e));
  return check_launch("attn_decode");
}

template <typename T>
static int dispatch_d(cudaStream_t s, const void* q, const void* k_new, const void* v_new,
                      void* k_cache, void* v_cache, const int64_t* pos, void* out, int64_t b,
                      int64_t h, int64_t max_len, int64_t d, int64_t ld_new, float scale) {
#define FERRITE_DECODE_D(DV) \
  if (d == DV) return launch<DV, T>(s, q, k_new, v_new, k_cache, v_cache, pos, out, b, h, max_len, ld_new, scale)
  FERRITE_DECODE_D(32);
  FERRITE_DECODE_D(64);
  FERRITE_DECODE_D(128);
  if constexpr (sizeof(T) == 2) FERRITE_DECODE_D(256);
#undef FERRITE_DECODE_D
  return fail(FERRITE_BAD_SHAPE, "attn_decode: head_dim %lld not in {32, 64, 128%s}", (long long)d,
              sizeof(T) == 2 ? ", 256" : "");
}

}  // namespace decode
}  // namespace ferrite

using namespace ferrite;
using namespace ferrite::decode;

extern "C" {

int ferrite_attn_decode(void* stream, const void* q, const void* k_new, const void* v_new,
                        void* k_cache, void* v_cache, const int64_t* pos, void* out, int64_t b,
                        int64_t h, int64_t max_len, int64_t d, int64_t ld_new, float scale,
                        int dtype) {
  if (b < 0 || h < 0 || max_len < 1 || d < 1)
    return fail(FERRITE_BAD_SHAPE, "attn_decode: bad sizes b=%lld h=%lld max_len=%lld d=%lld",
                (long long)b, (long long)h, (long long)max_len, (long long)d);
  if (ld_new < h * d)
    return fail(FERRITE_BAD_SHAPE, "attn_decode: ld_new %lld < h * d = %lld", (long long)ld_new,
                (long long)(h * d));
  if ((k_new == nullptr) != (v_new == nullptr))
    return fail(FERRITE_BAD_SHAPE, "attn_decode: k_new and v_new must both be given or both be null");
  if (dtype != FERRITE_BF16 && dtype != FERRITE_F16 && dtype != FERRITE_F32)
    return fail(FERRITE_UNSUPPORTED_DTYPE, "attn_decode: dtype %d", dtype);
  if (b * h > 0x7fffffffLL) return fail(FERRITE_BAD_SHAPE, "attn_decode: b * h above 2^31 - 1");
  if (b == 0 || h == 0) return FERRITE_OK;
  if (!q || !k_cache || !v_cache || !pos || !out) return fail(FERRITE_BAD_SHAPE, "attn_decode: null pointer");
  const int esz = dtype == FERRITE_F32 ? 4 : 2;
  auto mis = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) != 0; };
  if (mis(q) || mis(k_new) || mis(v_new) || mis(k_cache) || mis(v_cache) || mis(out) || (ld_new * esz) % 16 != 0)
    return fail(FERRITE_BAD_ALIGNMENT, "attn_decode: operands must be 16-byte aligned and ld_new * %d a multiple of 16", esz);
  if (int rc = injected_fault("attn_decode")) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == FERRITE_BF16)
    return dispatch_d<__nv_bfloat16>(s, q, k_new, v_new, k_cache, v_cache, pos, out, b, h, max_len, d, ld_new, scale);
  if (dtype == FERRITE_F16)
    return dispatch_d<__half>(s, q, k_new, v_new, k_cache, v_cache, pos, out, b, h, max_len, d, ld_new, scale);
  return dispatch_d<float>(s, q, k_new, v_new, k_cache, v_cache, pos, out, b, h, max_len, d, ld_new, scale);
}

// The cluster size ferrite_attn_decode launches with for b*h slices, without
// launching anything: the compiled rule above, with the lane groups of (d, dtype).
int ferrite_attn_decode_cluster(int64_t bh, int64_t max_len, int64_t d, int dtype, int64_t slots) {
  if (bh < 1 || max_len < 1 || slots < 1)
    return fail(FERRITE_BAD_SHAPE, "attn_decode_cluster: bh, max_len and slots must be positive"), -1;
  if (dtype != FERRITE_BF16 && dtype != FERRITE_F16 && dtype != FERRITE_F32)
    return fail(FERRITE_UNSUPPORTED_DTYPE, "attn_decode_cluster: dtype %d", dtype), -1;
  const int64_t epv = dtype == FERRITE_F32 ? 4 : 8;  // elements per 16-byte vector
  if (d % epv != 0 || d / epv > 32 || 32 % (d / epv) != 0)
    return fail(FERRITE_BAD_SHAPE, "attn_decode_cluster: head_dim %lld", (long long)d), -1;
  const int groups = kWarps * (int)(32 / (d / epv));
  return pick_cluster(bh, max_len, groups, slots);
}

}  // extern "C"
