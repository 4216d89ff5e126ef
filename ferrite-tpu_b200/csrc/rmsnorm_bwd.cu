// RMSNorm backward kernels (dh and the deterministic dw reduction) and their
// C-ABI entry points.
#include <mutex>

#include "rmsnorm_common.cuh"

namespace ferrite {
// The TMA-ring backward bounds its mbarrier waits; an expired wait is recorded in
// this translation unit's status word, which ferrite_device_status() polls.
FERRITE_DEFINE_STATUS_READER(status_rmsnorm)

namespace norm {

// ---------------------------------------------------------------------------
// backward
// ---------------------------------------------------------------------------

// Persistent backward.  Each row group walks rows r0, r0 + G, ... (G = row
// groups in the grid).  The next row's h, dy and dh_direct are loaded as raw
// 16-byte vectors before the current row is reduced, so one row's loads are
// always in flight while the previous row is reduced and written; the weight
// dw partial stays in registers for the whole kernel.
template <typename T, typename TW, bool HAS_DH, int VPT, int TPR, int CTA>
__global__ void __launch_bounds__(CTA, CTA <= 512 ? 2 : 1)
    rmsnorm_bwd_kernel(const T* __restrict__ h, const TW* __restrict__ w,
                       const T* __restrict__ dy, const T* __restrict__ dh_direct,
                       T* __restrict__ dh, float* __restrict__ partial,
                       int64_t rows, int dim, float eps) {
  constexpr int VE = Vec<T>::N;
  constexpr int RPC = CTA / TPR;
  __shared__ float red[CTA / 32 * 2 + 2];
  const int t = threadIdx.x % TPR;
  const int grp = threadIdx.x / TPR;
  const int nvec = dim / VE;
  const float inv_dim = 1.0f / (float)dim;
  pdl_launch_dependents();
  pdl_wait();

  float dwp[VPT][VE];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
#pragma unroll
    for (int j = 0; j < VE; ++j) dwp[i][j] = 0.f;
  }
  // The weight slice is re-read from L1 every row (16 KiB, shared by all rows).
  auto weights = [&](int i, float (&wv)[VE]) {
    const int vi = i * TPR + t;
    if (vi < nvec) {
      load_w<TW, VE>(w, (int64_t)vi * VE, wv);
    } else {
#pragma unroll
      for (int j = 0; j < VE; ++j) wv[j] = 0.f;
    }
  };

  const int64_t groups_total = (int64_t)gridDim.x * RPC;
  const int64_t first = (int64_t)blockIdx.x * RPC + grp;
  // Every thread runs the same number of iterations (the shared reduction needs
  // all of them); rows past the end are masked.
  const int64_t iters = (rows + groups_total - 1) / groups_total;
  uint4 ch[VPT], cg[VPT], cd[VPT];  // current row, raw
  uint4 nh[VPT], ng[VPT], nd[VPT];  // next row, raw
  auto load_row = [&](int64_t row, uint4 (&rh)[VPT], uint4 (&rg)[VPT], uint4 (&rd)[VPT]) {
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = i * TPR + t;
      if (row < rows && vi < nvec) {
        const int64_t e = row * (int64_t)dim + (int64_t)vi * VE;
        rh[i] = ld_stream_v4(h + e);
        rg[i] = ld_stream_v4(dy + e);
        if constexpr (HAS_DH) rd[i] = ld_stream_v4(dh_direct + e);
      } else {
        rh[i] = rg[i] = rd[i] = make_uint4(0, 0, 0, 0);
      }
    }
  };
  load_row(first, ch, cg, cd);
  for (int64_t it = 0; it < iters; ++it) {
    const int64_t row = first + it * groups_total;
    if (it + 1 < iters) load_row(row + groups_total, nh, ng, nd);
    float s2[2] = {0.f, 0.f};  // sum h^2, sum dy*w*h
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      float hv[VE], gv[VE], wv[VE];
      Vec<T>::to_f(ch[i], hv);
      Vec<T>::to_f(cg[i], gv);
      weights(i, wv);
#pragma unroll
      for (int j = 0; j < VE; ++j) {
        s2[0] = fmaf(hv[j], hv[j], s2[0]);
        s2[1] = fmaf(gv[j] * wv[j], hv[j], s2[1]);
      }
    }
    if constexpr (TPR > 32) {
      row_reduce<TPR, 2>(s2, red);
    } else {
      row_reduce<TPR, 2>(s2, nullptr);
    }
    const float inv = rsqrtf(s2[0] * inv_dim + eps);
    // mean(g * xhat) = inv * mean(dy*w*h)
    const float c = inv * s2[1] * inv_dim;
    if (row < rows) {
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int vi = i * TPR + t;
        if (vi < nvec) {
          float hv[VE], gv[VE], dd[VE], o[VE], wv[VE];
          Vec<T>::to_f(ch[i], hv);
          Vec<T>::to_f(cg[i], gv);
          weights(i, wv);
          if constexpr (HAS_DH) Vec<T>::to_f(cd[i], dd);
#pragma unroll
          for (int j = 0; j < VE; ++j) {
            const float xhat = hv[j] * inv;
            dwp[i][j] = fmaf(gv[j], xhat, dwp[i][j]);
            float v = inv * (gv[j] * wv[j] - xhat * c);
            if constexpr (HAS_DH) v += dd[j];
            o[j] = v;
          }
          st_v4(dh + row * (int64_t)dim + (int64_t)vi * VE, Vec<T>::from_f(o));
        }
      }
    }
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      ch[i] = nh[i];
      cg[i] = ng[i];
      cd[i] = nd[i];
    }
  }

  // Combine the RPC row groups of this CTA (fixed order), then write the CTA's
  // partial dw row.
  if constexpr (RPC > 1) {
    extern __shared__ float dwsm[];  // [RPC][dim]
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = i * TPR + t;
      if (vi < nvec) {
#pragma unroll
        for (int j = 0; j < VE; ++j) dwsm[grp * dim + vi * VE + j] = dwp[i][j];
      }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < dim; e += CTA) {
      float s = 0.f;
      for (int g = 0; g < RPC; ++g) s += dwsm[g * dim + e];
      partial[(int64_t)blockIdx.x * dim + e] = s;
    }
  } else {
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = i * TPR + t;
      if (vi < nvec) {
        float* p = partial + (int64_t)blockIdx.x * dim + (int64_t)vi * VE;
#pragma unroll
        for (int j = 0; j < VE; j += 4)
          *reinterpret_cast<float4*>(p + j) =
              make_float4(dwp[i][j], dwp[i][j + 1], dwp[i][j + 2], dwp[i][j + 3]);
      }
    }
  }
}

// TMA-fed backward for 16-bit rows of 256..4096 elements (dim = 8 x NC).  One
// producer warp streams each row's h, dy (and dh_direct) into a STAGES-deep
// shared-memory ring with 1-D bulk copies (cp.async.bulk, mbarrier
// complete_tx), so every CTA keeps STAGES-1 rows of loads in flight without
// spending registers on them; NC consumer threads each own 8 elements (one
// 16-byte vector) of the row, reduce the two row sums with warp shuffles and one
// named barrier, write dh and accumulate dw in registers.
template <typename T, typename TW, bool HAS_DH, int NC, int STAGES>
__global__ void __launch_bounds__(NC + 32, NC >= 512 ? 2 : 4)
    rmsnorm_bwd_tma_kernel(const T* __restrict__ h, const TW* __restrict__ w,
                           const T* __restrict__ dy, const T* __restrict__ dh_direct,
                           T* __restrict__ dh, float* __restrict__ partial, int64_t rows,
                           float eps) {
  constexpr int DIM = NC * 8;
  constexpr int ROW_BYTES = DIM * 2;
  constexpr int NT = HAS_DH ? 3 : 2;  // streamed tensors per row
  constexpr int NW = NC / 32;         // consumer warps
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * NT * ROW_BYTES);
  uint64_t* empty = full + STAGES;
  float* red = reinterpret_cast<float*>(empty + STAGES);  // [2][NW][2]
  volatile int* abort = reinterpret_cast<volatile int*>(red + 2 * NW * 2);
  const int tid = threadIdx.x;
  if (tid == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], NW);
    }
    *abort = 0;
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();
  pdl_wait();
  const int64_t first = blockIdx.x, stride = gridDim.x;
  const int64_t my_rows = first < rows ? (rows - first + stride - 1) / stride : 0;
  auto stage = [&](int s, int t) { return smem + (s * NT + t) * ROW_BYTES; };

  if (tid >= NC) {
    // ---------------------------------------------------------------- producer
    if (tid == NC) {
      for (int64_t it = 0; it < my_rows; ++it) {
        const int s = (int)(it % STAGES);
        if (!mbar_wait(&empty[s], (uint32_t)((it / STAGES) & 1) ^ 1u, abort, 40)) break;
        const int64_t off = (first + it * stride) * DIM;
        mbar_arrive_expect_tx(&full[s], NT * ROW_BYTES);
        bulk_load(stage(s, 0), h + off, ROW_BYTES, &full[s]);
        bulk_load(stage(s, 1), dy + off, ROW_BYTES, &full[s]);
        if constexpr (HAS_DH) bulk_load(stage(s, 2), dh_direct + off, ROW_BYTES, &full[s]);
      }
    }
    return;
  }
  // ------------------------------------------------------------------ consumers
  const int warp = tid >> 5, lane = tid & 31;
  constexpr int VE = 8;
  float wv[VE], dwp[VE];
  load_w<TW, VE>(w, (int64_t)tid * VE, wv);
#pragma unroll
  for (int j = 0; j < VE; ++j) dwp[j] = 0.f;
  const float inv_dim = 1.0f / (float)DIM;
  for (int64_t it = 0; it < my_rows; ++it) {
    const int s = (int)(it % STAGES);
    if (!mbar_wait(&full[s], (uint32_t)((it / STAGES) & 1), abort, 41)) break;
    float hv[VE], gv[VE], dd[VE];
    Vec<T>::to_f(*reinterpret_cast<const uint4*>(stage(s, 0) + tid * 16), hv);
    Vec<T>::to_f(*reinterpret_cast<const uint4*>(stage(s, 1) + tid * 16), gv);
    if constexpr (HAS_DH) Vec<T>::to_f(*reinterpret_cast<const uint4*>(stage(s, 2) + tid * 16), dd);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);  // this warp is done with the slot
    float a = 0.f, b = 0.f;  // sum h^2, sum dy*w*h
#pragma unroll
    for (int j = 0; j < VE; ++j) {
      a = fmaf(hv[j], hv[j], a);
      b = fmaf(gv[j] * wv[j], hv[j], b);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      a += __shfl_xor_sync(0xffffffffu, a, o);
      b += __shfl_xor_sync(0xffffffffu, b, o);
    }
    float* rb = red + (it & 1) * NW * 2;
    if (lane == 0) {
      rb[warp * 2] = a;
      rb[warp * 2 + 1] = b;
    }
    named_barrier(1, NC);
    a = 0.f;
    b = 0.f;
#pragma unroll
    for (int q = 0; q < NW; ++q) {
      a += rb[q * 2];
      b += rb[q * 2 + 1];
    }
    const float inv = rsqrtf(a * inv_dim + eps);
    const float c = inv * b * inv_dim;  // mean(g * xhat)
    float o[VE];
#pragma unroll
    for (int j = 0; j < VE; ++j) {
      const float xhat = hv[j] * inv;
      dwp[j] = fmaf(gv[j], xhat, dwp[j]);
      float v = inv * (gv[j] * wv[j] - xhat * c);
      if constexpr (HAS_DH) v += dd[j];
      o[j] = v;
    }
    st_v4(dh + (first + it * stride) * DIM + (int64_t)tid * VE, Vec<T>::from_f(o));
  }
  float* p = partial + (int64_t)blockIdx.x * DIM + (int64_t)tid * VE;
  *reinterpret_cast<float4*>(p) = make_float4(dwp[0], dwp[1], dwp[2], dwp[3]);
  *reinterpret_cast<float4*>(p + 4) = make_float4(dwp[4], dwp[5], dwp[6], dwp[7]);
}

template <typename T, typename TW, bool HAS_DH>
__global__ void __launch_bounds__(256)
    rmsnorm_bwd_scalar(const T* __restrict__ h, const TW* __restrict__ w,
                       const T* __restrict__ dy, const T* __restrict__ dh_direct,
                       T* __restrict__ dh, float* __restrict__ partial,
                       int64_t rows, int dim, float eps) {
  // Persistent grid; each warp walks rows, each lane owns columns lane+32k.
  // partial layout: [gridDim.x * 8][dim] (one row per warp).
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  const int64_t gw = (int64_t)blockIdx.x * 8 + wib;
  const int64_t nw = (int64_t)gridDim.x * 8;
  pdl_launch_dependents();
  pdl_wait();
  float* my = partial + gw * dim;
  for (int j = lane; j < dim; j += 32) my[j] = 0.f;
  const float inv_dim = 1.0f / (float)dim;
  for (int64_t row = gw; row < rows; row += nw) {
    const int64_t base = row * (int64_t)dim;
    float a = 0.f, b = 0.f;
    for (int j = lane; j < dim; j += 32) {
      const float hv = DT<T>::to_f(h[base + j]);
      const float g = DT<T>::to_f(dy[base + j]) * DT<TW>::to_f(w[j]);
      a = fmaf(hv, hv, a);
      b = fmaf(g, hv, b);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      a += __shfl_xor_sync(0xffffffffu, a, off);
      b += __shfl_xor_sync(0xffffffffu, b, off);
    }
    const float inv = rsqrtf(a * inv_dim + eps);
    const float c = inv * b * inv_dim;
    for (int j = lane; j < dim; j += 32) {
      const float hv = DT<T>::to_f(h[base + j]);
      const float dyv = DT<T>::to_f(dy[base + j]);
      const float xhat = hv * inv;
      const float g = dyv * DT<TW>::to_f(w[j]);
      float v = inv * (g - xhat * c);
      if constexpr (HAS_DH) v += DT<T>::to_f(dh_direct[base + j]);
      dh[base + j] = DT<T>::from_f(v);
      my[j] = fmaf(dyv, xhat, my[j]);
    }
  }
}

// dw = sum of the nparts partial rows, in a fixed order (bitwise deterministic).
// CTA = 16 columns x 32 row groups; each thread issues all of its partial loads
// (up to 16, rows ty, ty + 32, ...) before summing them in order, so the
// reduction costs one round of L2 latency instead of one per load; the 32 row
// groups are then added in order through shared memory.
constexpr int kDwCols = 16;
template <typename TW>
__global__ void __launch_bounds__(512)
    dw_reduce_kernel(const float* __restrict__ partial, TW* __restrict__ dw,
                     int nparts, int dim) {
  __shared__ float sm[32][kDwCols + 1];
  const int tx = threadIdx.x % kDwCols, ty = threadIdx.x / kDwCols;
  const int e = blockIdx.x * kDwCols + tx;
  pdl_launch_dependents();
  pdl_wait();
  float acc = 0.f;
  if (e < dim) {
    for (int p0 = 0; p0 < nparts; p0 += 32 * 16) {
      float v[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const int p = p0 + ty + 32 * k;
        v[k] = p < nparts ? partial[(int64_t)p * dim + e] : 0.f;
      }
#pragma unroll
      for (int k = 0; k < 16; ++k) acc += v[k];
    }
  }
  sm[ty][tx] = acc;
  __syncthreads();
  if (ty == 0 && e < dim) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 32; ++k) t += sm[k][tx];
    dw[e] = DT<TW>::from_f(t);
  }
}

// Persistent grid of the backward kernel and the resulting partial count.
struct BwdPlan {
  Cfg c;
  int grid;
  int nparts;  // rows of the partial-sum workspace
  int smem;    // dynamic shared memory bytes
  void* tma_kernel = nullptr;  // TMA-fed kernel when set (16-bit rows of 256..4096)
  int tma_threads = 0;
};

// Backward CTA size: at least 512 threads so that one CTA keeps enough loads in
// flight and the persistent grid (and with it the dw partial workspace) stays
// small.
constexpr int bwd_cta(int tpr) { return tpr >= 512 ? tpr : 512; }

template <typename T, typename TW, bool HAS_DH, int VPT, int TPR>
static void* bwd_kernel_ptr() {
  return (void*)rmsnorm_bwd_kernel<T, TW, HAS_DH, VPT, TPR, bwd_cta(TPR)>;
}

template <typename T, typename TW, bool HAS_DH, int VPT>
static void* bwd_ptr_tpr(int tpr) {
#define BWD_CASE(N)                                                              \
  case N:                                                                        \
    if constexpr ((VPT == 1) || (VPT == 2 && N >= 64) || (VPT == 4 && N >= 256)) \
      return bwd_kernel_ptr<T, TW, HAS_DH, VPT, N>();                            \
    break;
  switch (tpr) {
    BWD_CASE(4) BWD_CASE(8) BWD_CASE(16) BWD_CASE(32) BWD_CASE(64) BWD_CASE(128)
    BWD_CASE(256) BWD_CASE(512) BWD_CASE(1024)
  }
#undef BWD_CASE
  return nullptr;
}

template <typename T, typename TW, bool HAS_DH>
static void* bwd_ptr(const Cfg& c) {
  switch (c.vpt) {
    case 1: return bwd_ptr_tpr<T, TW, HAS_DH, 1>(c.tpr);
    case 2: return bwd_ptr_tpr<T, TW, HAS_DH, 2>(c.tpr);
    case 4: return bwd_ptr_tpr<T, TW, HAS_DH, 4>(c.tpr);
  }
  return nullptr;
}

constexpr int kTmaStages = 4;

template <typename T, typename TW, bool HAS_DH, int NC>
static void* tma_kernel_ptr() {
  return (void*)rmsnorm_bwd_tma_kernel<T, TW, HAS_DH, NC, kTmaStages>;
}

// TMA-fed plan for 16-bit rows whose length is 8 x {32, 64, 128, 256, 512}.
template <typename T, typename TW, bool HAS_DH>
static bool plan_bwd_tma(BwdPlan& p, int64_t rows, int64_t dim, const void* const* ptrs,
                         int nptr, int device) {
  if constexpr (sizeof(T) != 2) {
    return false;
  } else {
    if (env_int("FERRITE_RMSNORM_BWD_TMA", 1) == 0) return false;
    for (int i = 0; i < nptr; ++i)
      if (ptrs[i] && (reinterpret_cast<uintptr_t>(ptrs[i]) & 15u)) return false;
    void* k = nullptr;
    switch (dim) {
      case 256: k = tma_kernel_ptr<T, TW, HAS_DH, 32>(); break;
      case 512: k = tma_kernel_ptr<T, TW, HAS_DH, 64>(); break;
      case 1024: k = tma_kernel_ptr<T, TW, HAS_DH, 128>(); break;
      case 2048: k = tma_kernel_ptr<T, TW, HAS_DH, 256>(); break;
      case 4096: k = tma_kernel_ptr<T, TW, HAS_DH, 512>(); break;
      default: return false;
    }
    const int nc = (int)(dim / 8);
    const int nt = HAS_DH ? 3 : 2;
    const int smem = kTmaStages * nt * (int)dim * 2 + 2 * kTmaStages * 8 + 2 * (nc / 32) * 2 * 4 + 16;
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return false;
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k, nc + 32, smem) != cudaSuccess || occ < 1)
      return false;
    occ = std::min(occ, 8);
    p.grid = (int)std::max<int64_t>(1, std::min<int64_t>(rows, (int64_t)num_sms(device) * occ));
    p.nparts = p.grid;
    p.smem = smem;
    p.tma_kernel = k;
    p.tma_threads = nc + 32;
    return true;
  }
}

template <typename T, typename TW, bool HAS_DH>
static BwdPlan plan_bwd(int64_t rows, int64_t dim, const void* const* ptrs,
                        int nptr, int device) {
  BwdPlan p{};
  if (plan_bwd_tma<T, TW, HAS_DH>(p, rows, dim, ptrs, nptr, device)) return p;
  p.c = pick(dim, sizeof(T), ptrs, nptr, true);
  const int sms = num_sms(device);
  if (p.c.vec) {
    const int CTA = bwd_cta(p.c.tpr);
    const int RPC = CTA / p.c.tpr;
    p.smem = RPC > 1 ? RPC * (int)dim * 4 : 0;
    void* k = bwd_ptr<T, TW, HAS_DH>(p.c);
    int occ = 0;
    if (k == nullptr || p.smem > 200 * 1024) {
      p.c.vec = false;
    } else {
      if (p.smem > 48 * 1024)
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, p.smem);
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k, CTA, p.smem) !=
              cudaSuccess ||
          occ < 1)
        occ = 1;
      occ = std::min(occ, env_int("FERRITE_RMSNORM_BWD_CTAS_PER_SM", occ));
      occ = std::max(1, std::min(occ, 4));
      const int64_t groups = (rows + RPC - 1) / RPC;
      p.grid = (int)std::max<int64_t>(1, std::min<int64_t>(groups, (int64_t)sms * occ));
      p.nparts = p.grid;
    }
  }
  if (!p.c.vec) {
    p.grid = (int)std::max<int64_t>(1, std::min<int64_t>((rows + 7) / 8, sms));
    p.nparts = p.grid * 8;
    p.smem = 0;
  }
  return p;
}

static int launch_tma(const BwdPlan& p, cudaStream_t s, const void* h, const void* w,
                      const void* dy, const void* dhd, void* dh, float* part, int64_t rows,
                      float eps) {
  void* args[] = {&h, &w, &dy, &dhd, &dh, &part, &rows, &eps};
  cudaError_t e = launch_k(p.tma_kernel, dim3(p.grid), dim3(p.tma_threads), p.smem, s, args);
  if (e != cudaSuccess)
    return fail(FERRITE_LAUNCH_FAILED, "rmsnorm_bwd (tma): %s", cudaGetErrorString(e));
  return FERRITE_OK;
}

template <typename T, typename TW, bool HAS_DH>
static int run_bwd(cudaStream_t s, const void* h, const void* w, const void* dy,
                   const void* dhd, void* dh, void* dw, void* ws,
                   size_t ws_bytes, int64_t rows, int64_t dim, float eps) {
  const int dev = current_device();
  const void* ptrs[5] = {h, dy, HAS_DH ? dhd : nullptr, dh, w};
  BwdPlan p = plan_bwd<T, TW, HAS_DH>(rows, dim, ptrs, 5, dev);
  const size_t need = (size_t)p.nparts * (size_t)dim * sizeof(float);
  if (ws == nullptr || ws_bytes < need)
    return fail(FERRITE_WORKSPACE_TOO_SMALL,
                "rmsnorm_bwd: workspace %zu bytes < %zu needed", ws_bytes, need);
  if ((reinterpret_cast<uintptr_t>(ws) & 15u) != 0)
    return fail(FERRITE_BAD_ALIGNMENT, "rmsnorm_bwd: workspace not 16-byte aligned");
  if (p.tma_kernel) {
    if (int rc = launch_tma(p, s, h, w, dy, dhd, dh, (float*)ws, rows, eps)) return rc;
  } else if (p.c.vec) {
    void* k = bwd_ptr<T, TW, HAS_DH>(p.c);
    const int CTA = bwd_cta(p.c.tpr);
    int dimi = (int)dim;
    const T* hp = (const T*)h;
    const TW* wp = (const TW*)w;
    const T* dyp = (const T*)dy;
    const T* dhdp = (const T*)dhd;
    T* dhp = (T*)dh;
    float* part = (float*)ws;
    void* args[] = {&hp, &wp, &dyp, &dhdp, &dhp, &part, &rows, &dimi, &eps};
    cudaError_t e = launch_k(k, dim3(p.grid), dim3(CTA), p.smem, s, args);
    if (e != cudaSuccess)
      return fail(FERRITE_LAUNCH_FAILED, "rmsnorm_bwd: %s", cudaGetErrorString(e));
  } else {
    cudaError_t e = launch_pdl(rmsnorm_bwd_scalar<T, TW, HAS_DH>, dim3(p.grid), dim3(256), 0, s,
                               (const T*)h, (const TW*)w, (const T*)dy, (const T*)dhd, (T*)dh,
                               (float*)ws, rows, (int)dim, eps);
    if (e != cudaSuccess) return fail(FERRITE_LAUNCH_FAILED, "rmsnorm_bwd: %s", cudaGetErrorString(e));
  }
  if (int rc = check_launch("rmsnorm_bwd")) return rc;
  cudaError_t e = launch_pdl(dw_reduce_kernel<TW>, dim3((unsigned)((dim + kDwCols - 1) / kDwCols)), dim3(512), 0, s,
                             (const float*)ws, (TW*)dw, p.nparts, (int)dim);
  if (e != cudaSuccess) return fail(FERRITE_LAUNCH_FAILED, "rmsnorm_dw_reduce: %s", cudaGetErrorString(e));
  return check_launch("rmsnorm_dw_reduce");
}


// ---------------------------------------------------------------------------
// Allocation-free variant (ferrite_rmsnorm_bwd_noalloc)
// ---------------------------------------------------------------------------
//
// Some callers cannot hand the backward a workspace: a host framework that owns
// all device memory and gives its kernels no scratch allocator, or a runtime that
// sizes its device arena once at start-up and allows no allocation afterwards
// (cudaMalloc / cudaFree can synchronise the device and are not stream-ordered).
// For them the dw partial sums live in a library-owned, file-scope device array
// of fixed size instead of a caller workspace.  Every GPU that loads the library
// holds this array (4 MiB) until the process exits.

// Capacity of the library-owned dw partial buffer, in floats (4 MiB per device).
constexpr int64_t kNoAllocPartialFloats = int64_t(1) << 20;
// Largest row length the allocation-free variant accepts: its scalar plan needs
// 8 partial rows per CTA and at least one CTA.
constexpr int64_t kNoAllocMaxDim = kNoAllocPartialFloats / 8;

static __device__ __align__(256) float g_noalloc_partials[kNoAllocPartialFloats];

namespace {
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[64] = {nullptr};
}  // namespace

// Device address of g_noalloc_partials on the current device, and that device.
// In host code the array's name is only a host-side stand-in, so the address is
// looked up once per device with cudaGetSymbolAddress (that device current) and
// cached.  The cache belongs to the device's primary context in this process: a
// process that calls cudaDeviceReset must not call the allocation-free entry
// point on that device afterwards.
static int noalloc_partials(int* device, float** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return fail(FERRITE_LAUNCH_FAILED, "rmsnorm_bwd_noalloc: cudaGetDevice failed: %s",
                cudaGetErrorString(e));
  if (dev < 0 || dev >= 64)
    return fail(FERRITE_LAUNCH_FAILED, "rmsnorm_bwd_noalloc: device ordinal %d beyond the 64 the address cache holds", dev);
  *device = dev;
  float* p = __atomic_load_n(&g_noalloc_ptr[dev], __ATOMIC_ACQUIRE);
  if (p == nullptr) {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    p = g_noalloc_ptr[dev];
    if (p == nullptr) {
      void* addr = nullptr;
      e = cudaGetSymbolAddress(&addr, g_noalloc_partials);
      if (e != cudaSuccess || addr == nullptr)
        return fail(FERRITE_LAUNCH_FAILED, "rmsnorm_bwd_noalloc: cudaGetSymbolAddress failed: %s",
                    cudaGetErrorString(e));
      p = static_cast<float*>(addr);
      __atomic_store_n(&g_noalloc_ptr[dev], p, __ATOMIC_RELEASE);
    }
  }
  *out = p;
  return FERRITE_OK;
}

template <typename T, typename TW, bool HAS_DH>
static int run_bwd_noalloc(cudaStream_t s, const void* h, const void* w, const void* dy,
                           const void* dhd, void* dh, void* dw, int64_t rows, int64_t dim,
                           float eps) {
  int dev = 0;
  float* part = nullptr;
  if (int rc = noalloc_partials(&dev, &part)) return rc;
  const void* ptrs[5] = {h, dy, HAS_DH ? dhd : nullptr, dh, w};
  BwdPlan p = plan_bwd<T, TW, HAS_DH>(rows, dim, ptrs, 5, dev);
  // Fit the partial rows into the fixed buffer (the persistent kernels accept
  // any grid size; a smaller grid only means more rows per CTA).
  const int64_t max_rows = kNoAllocPartialFloats / dim;
  if (p.tma_kernel) {
    p.grid = (int)std::max<int64_t>(1, std::min<int64_t>(p.grid, max_rows));
    p.nparts = p.grid;
  } else if (p.c.vec) {
    p.grid = (int)std::max<int64_t>(1, std::min<int64_t>(p.grid, max_rows));
    p.nparts = p.grid;
  } else {
    p.grid = (int)std::max<int64_t>(1, std::min<int64_t>(p.grid, max_rows / 8));
    p.nparts = p.grid * 8;
  }
  if ((int64_t)p.nparts * dim > kNoAllocPartialFloats)
    return fail(FERRITE_BAD_SHAPE, "rmsnorm_bwd_noalloc: dim %lld needs more than the %lld-float buffer",
                (long long)dim, (long long)kNoAllocPartialFloats);
  if (p.tma_kernel) {
    if (int rc = launch_tma(p, s, h, w, dy, dhd, dh, part, rows, eps)) return rc;
  } else if (p.c.vec) {
    void* k = bwd_ptr<T, TW, HAS_DH>(p.c);
    const int CTA = bwd_cta(p.c.tpr);
    int dimi = (int)dim;
    const T* hp = (const T*)h;
    const TW* wp = (const TW*)w;
    const T* dyp = (const T*)dy;
    const T* dhdp = (const T*)dhd;
    T* dhp = (T*)dh;
    void* args[] = {&hp, &wp, &dyp, &dhdp, &dhp, &part, &rows, &dimi, &eps};
    cudaError_t e = launch_k(k, dim3(p.grid), dim3(CTA), p.smem, s, args);
    if (e != cudaSuccess)
      return fail(FERRITE_LAUNCH_FAILED, "rmsnorm_bwd_noalloc: %s", cudaGetErrorString(e));
  } else {
    cudaError_t e = launch_pdl(rmsnorm_bwd_scalar<T, TW, HAS_DH>, dim3(p.grid), dim3(256), 0, s,
                               (const T*)h, (const TW*)w, (const T*)dy, (const T*)dhd, (T*)dh, part, rows, (int)dim, eps);
    if (e != cudaSuccess) return fail(FERRITE_LAUNCH_FAILED, "rmsnorm_bwd_noalloc: %s", cudaGetErrorString(e));
  }
  if (int rc = check_launch("rmsnorm_bwd_noalloc")) return rc;
  cudaError_t e = launch_pdl(dw_reduce_kernel<TW>, dim3((unsigned)((dim + kDwCols - 1) / kDwCols)), dim3(512), 0, s,
                             (const float*)part, (TW*)dw, p.nparts, (int)dim);
  if (e != cudaSuccess) return fail(FERRITE_LAUNCH_FAILED, "rmsnorm_bwd_noalloc dw_reduce: %s", cudaGetErrorString(e));
  return check_launch("rmsnorm_bwd_noalloc_dw_reduce");
}

}  // namespace norm
}  // namespace ferrite

using namespace ferrite;
using namespace ferrite::norm;

extern "C" {

size_t ferrite_rmsnorm_bwd_workspace_size(int64_t rows, int64_t dim) {
  if (dim <= 0) return 16;
  return (size_t)max_parts(rows, current_device()) * (size_t)dim * sizeof(float);
}

int ferrite_rmsnorm_bwd(void* stream, const void* h, const void* w,
                        const void* dy, const void* dh_direct, void* dh,
                        void* dw, void* workspace, size_t workspace_bytes,
                        int64_t rows, int64_t dim, float eps, int dtype,
                        int w_dtype) {
  if (int rc = check_common("rmsnorm_bwd", rows, dim, dtype, w_dtype)) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  if (!dw) return fail(FERRITE_BAD_SHAPE, "rmsnorm_bwd: null dw");
  if (rows == 0) {
    cudaError_t e = cudaMemsetAsync(dw, 0, dim * (w_dtype == FERRITE_F32 ? 4 : 2), s);
    return e == cudaSuccess ? FERRITE_OK
                            : fail(FERRITE_LAUNCH_FAILED, "rmsnorm_bwd: memset");
  }
  if (!h || !w || !dy || !dh) return fail(FERRITE_BAD_SHAPE, "rmsnorm_bwd: null pointer");
  const bool has = dh_direct != nullptr;
#define CALL(T, TW)                                                                  \
  (has ? run_bwd<T, TW, true>(s, h, w, dy, dh_direct, dh, dw, workspace,             \
                              workspace_bytes, rows, dim, eps)                       \
       : run_bwd<T, TW, false>(s, h, w, dy, dh_direct, dh, dw, workspace,            \
                               workspace_bytes, rows, dim, eps))
  if (dtype == FERRITE_BF16 && w_dtype == FERRITE_F32) return CALL(__nv_bfloat16, float);
  if (dtype == FERRITE_BF16 && w_dtype == FERRITE_BF16) return CALL(__nv_bfloat16, __nv_bfloat16);
  if (dtype == FERRITE_F32 && w_dtype == FERRITE_F32) return CALL(float, float);
  if (dtype == FERRITE_F16 && w_dtype == FERRITE_F32) return CALL(__half, float);
#undef CALL
  return fail(FERRITE_UNSUPPORTED_DTYPE, "rmsnorm_bwd: dtype");
}


// Allocation-free RMSNorm backward; see the section comment above and the
// declaration in ferrite_b200.h.  The first call on a device looks up the
// buffer's device address (cudaGetSymbolAddress) with that device current;
// make that first call before any stream capture.
int ferrite_rmsnorm_bwd_noalloc(void* stream, const void* h, const void* w, const void* dy,
                                const void* dh_direct, void* dh, void* dw, int64_t rows,
                                int64_t dim, float eps, int dtype, int w_dtype) {
  if (int rc = check_common("rmsnorm_bwd_noalloc", rows, dim, dtype, w_dtype)) return rc;
  if (dim > kNoAllocMaxDim)
    return fail(FERRITE_BAD_SHAPE,
                "rmsnorm_bwd_noalloc: dim %lld exceeds the allocation-free maximum %lld",
                (long long)dim, (long long)kNoAllocMaxDim);
  cudaStream_t s = (cudaStream_t)stream;
  if (!dw) return fail(FERRITE_BAD_SHAPE, "rmsnorm_bwd_noalloc: null dw");
  if (rows == 0) {
    cudaError_t e = cudaMemsetAsync(dw, 0, dim * (w_dtype == FERRITE_F32 ? 4 : 2), s);
    return e == cudaSuccess ? FERRITE_OK
                            : fail(FERRITE_LAUNCH_FAILED, "rmsnorm_bwd_noalloc: memset");
  }
  if (!h || !w || !dy || !dh) return fail(FERRITE_BAD_SHAPE, "rmsnorm_bwd_noalloc: null pointer");
  const bool has = dh_direct != nullptr;
#define CALL(T, TW)                                                                         \
  (has ? run_bwd_noalloc<T, TW, true>(s, h, w, dy, dh_direct, dh, dw, rows, dim, eps)       \
       : run_bwd_noalloc<T, TW, false>(s, h, w, dy, dh_direct, dh, dw, rows, dim, eps))
  if (dtype == FERRITE_BF16 && w_dtype == FERRITE_F32) return CALL(__nv_bfloat16, float);
  if (dtype == FERRITE_BF16 && w_dtype == FERRITE_BF16) return CALL(__nv_bfloat16, __nv_bfloat16);
  if (dtype == FERRITE_F32 && w_dtype == FERRITE_F32) return CALL(float, float);
  if (dtype == FERRITE_F16 && w_dtype == FERRITE_F32) return CALL(__half, float);
#undef CALL
  return fail(FERRITE_UNSUPPORTED_DTYPE, "rmsnorm_bwd_noalloc: dtype");
}

}  // extern "C"
