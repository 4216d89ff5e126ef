// Fused residual-add + RMSNorm forward kernels and their C-ABI entry points.
#include "rmsnorm_common.cuh"

namespace ferrite {
namespace norm {

// ---------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------

template <typename T, typename TW, bool ADD, int VPT, int TPR, int CTA>
__global__ void __launch_bounds__(CTA)
    rmsnorm_fwd_kernel(const T* __restrict__ x, const T* __restrict__ r,
                       const TW* __restrict__ w, T* __restrict__ h_out,
                       T* __restrict__ y, int64_t rows, int dim, float eps) {
  constexpr int VE = Vec<T>::N;
  constexpr int RPC = CTA / TPR;  // rows per CTA
  __shared__ float red[CTA / 32 * 1 + 1];
  const int t = threadIdx.x % TPR;
  const int64_t row = (int64_t)blockIdx.x * RPC + threadIdx.x / TPR;
  const bool active = row < rows;
  const int nvec = dim / VE;
  const int64_t base = row * (int64_t)dim;
  pdl_launch_dependents();
  pdl_wait();

  float hv[VPT][VE];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = i * TPR + t;
    if (active && vi < nvec) {
      const int64_t e = base + (int64_t)vi * VE;
      Vec<T>::to_f(ld_stream_v4(x + e), hv[i]);
      if constexpr (ADD) {
        float rv[VE];
        Vec<T>::to_f(ld_stream_v4(r + e), rv);
#pragma unroll
        for (int j = 0; j < VE; ++j) hv[i][j] += rv[j];
        st_v4(h_out + e, Vec<T>::from_f(hv[i]));
      }
#pragma unroll
      for (int j = 0; j < VE; ++j) ss = fmaf(hv[i][j], hv[i][j], ss);
    }
  }
  float tot[1] = {ss};
  if constexpr (TPR > 32) {
    row_reduce<TPR, 1>(tot, red);
  } else {
    row_reduce<TPR, 1>(tot, nullptr);
  }
  const float inv = rsqrtf(tot[0] * (1.0f / (float)dim) + eps);
  if (!active) return;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = i * TPR + t;
    if (vi < nvec) {
      float wv[VE];
      load_w<TW, VE>(w, (int64_t)vi * VE, wv);
      float o[VE];
#pragma unroll
      for (int j = 0; j < VE; ++j) o[j] = hv[i][j] * inv * wv[j];
      st_v4(y + base + (int64_t)vi * VE, Vec<T>::from_f(o));
    }
  }
}

// Scalar fallback (any dim, any alignment): one warp per row, two passes over
// global memory (the second pass re-reads from L1/L2).
template <typename T, typename TW, bool ADD>
__global__ void __launch_bounds__(256)
    rmsnorm_fwd_scalar(const T* __restrict__ x, const T* __restrict__ r,
                       const TW* __restrict__ w, T* __restrict__ h_out,
                       T* __restrict__ y, int64_t rows, int dim, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  pdl_launch_dependents();
  if (row >= rows) return;
  pdl_wait();
  const int64_t base = row * (int64_t)dim;
  float ss = 0.f;
  for (int j = lane; j < dim; j += 32) {
    float hv = DT<T>::to_f(x[base + j]);
    if constexpr (ADD) {
      hv += DT<T>::to_f(r[base + j]);
      h_out[base + j] = DT<T>::from_f(hv);
    }
    ss = fmaf(hv, hv, ss);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float inv = rsqrtf(ss * (1.0f / (float)dim) + eps);
  for (int j = lane; j < dim; j += 32) {
    float hv = DT<T>::to_f(x[base + j]);
    if constexpr (ADD) hv += DT<T>::to_f(r[base + j]);
    y[base + j] = DT<T>::from_f(hv * inv * DT<TW>::to_f(w[j]));
  }
}

template <typename T, typename TW, bool ADD, int VPT, int TPR>
static int launch_fwd_t(cudaStream_t s, const void* x, const void* r,
                        const void* w, void* h, void* y, int64_t rows, int dim,
                        float eps) {
  constexpr int CTA = TPR >= 256 ? TPR : 256;
  constexpr int RPC = CTA / TPR;
  const int64_t grid = (rows + RPC - 1) / RPC;
  if (grid > 0x7fffffff) return fail(FERRITE_BAD_SHAPE, "rmsnorm: too many rows");
  cudaError_t e = launch_pdl(rmsnorm_fwd_kernel<T, TW, ADD, VPT, TPR, CTA>, dim3((unsigned)grid), dim3(CTA), 0, s,
                             (const T*)x, (const T*)r, (const TW*)w, (T*)h, (T*)y, rows, dim, eps);
  if (e != cudaSuccess) return fail(FERRITE_LAUNCH_FAILED, "rmsnorm_fwd: launch failed: %s", cudaGetErrorString(e));
  return check_launch("rmsnorm_fwd");
}

template <typename T, typename TW, bool ADD, int VPT>
static int dispatch_fwd_tpr(int tpr, cudaStream_t s, const void* x,
                            const void* r, const void* w, void* h, void* y,
                            int64_t rows, int dim, float eps) {
#define FWD_CASE(N)                                                                  \
  case N:                                                                            \
    if constexpr ((VPT == 1) || (VPT == 2 && N >= 64) || (VPT == 4 && N >= 256))     \
      return launch_fwd_t<T, TW, ADD, VPT, N>(s, x, r, w, h, y, rows, dim, eps);     \
    break;
  switch (tpr) {
    FWD_CASE(4) FWD_CASE(8) FWD_CASE(16) FWD_CASE(32) FWD_CASE(64) FWD_CASE(128)
    FWD_CASE(256) FWD_CASE(512) FWD_CASE(1024)
  }
#undef FWD_CASE
  return fail(FERRITE_BAD_SHAPE, "rmsnorm: bad threads-per-row %d", tpr);
}

template <typename T, typename TW, bool ADD>
static int run_fwd(cudaStream_t s, const void* x, const void* r, const void* w,
                   void* h, void* y, int64_t rows, int64_t dim, float eps) {
  const void* ptrs[5] = {x, ADD ? r : nullptr, ADD ? h : nullptr, y, w};
  Cfg c = pick(dim, sizeof(T), ptrs, 5, false);
  if (!c.vec) {
    const int64_t grid = (rows + 7) / 8;
    cudaError_t e = launch_pdl(rmsnorm_fwd_scalar<T, TW, ADD>, dim3((unsigned)grid), dim3(256), 0, s,
                               (const T*)x, (const T*)r, (const TW*)w, (T*)h, (T*)y, rows, (int)dim, eps);
    if (e != cudaSuccess) return fail(FERRITE_LAUNCH_FAILED, "rmsnorm_fwd_scalar: launch failed: %s", cudaGetErrorString(e));
    return check_launch("rmsnorm_fwd_scalar");
  }
  switch (c.vpt) {
    case 1: return dispatch_fwd_tpr<T, TW, ADD, 1>(c.tpr, s, x, r, w, h, y, rows, (int)dim, eps);
    case 2: return dispatch_fwd_tpr<T, TW, ADD, 2>(c.tpr, s, x, r, w, h, y, rows, (int)dim, eps);
    case 4: return dispatch_fwd_tpr<T, TW, ADD, 4>(c.tpr, s, x, r, w, h, y, rows, (int)dim, eps);
  }
  return fail(FERRITE_BAD_SHAPE, "rmsnorm: bad vectors-per-thread");
}

}  // namespace norm
}  // namespace ferrite

using namespace ferrite;
using namespace ferrite::norm;

extern "C" {

int ferrite_rmsnorm_fwd(void* stream, const void* x, const void* w, void* y,
                        int64_t rows, int64_t dim, float eps, int dtype,
                        int w_dtype) {
  if (int rc = check_common("rmsnorm_fwd", rows, dim, dtype, w_dtype)) return rc;
  if (rows == 0) return FERRITE_OK;
  if (!x || !w || !y) return fail(FERRITE_BAD_SHAPE, "rmsnorm_fwd: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
#define CALL(T, TW, ADD) run_fwd<T, TW, ADD>(s, x, nullptr, w, nullptr, y, rows, dim, eps)
  if (dtype == FERRITE_BF16 && w_dtype == FERRITE_F32) return CALL(__nv_bfloat16, float, false);
  if (dtype == FERRITE_BF16 && w_dtype == FERRITE_BF16) return CALL(__nv_bfloat16, __nv_bfloat16, false);
  if (dtype == FERRITE_F32 && w_dtype == FERRITE_F32) return CALL(float, float, false);
  if (dtype == FERRITE_F16 && w_dtype == FERRITE_F32) return CALL(__half, float, false);
#undef CALL
  return fail(FERRITE_UNSUPPORTED_DTYPE, "rmsnorm_fwd: dtype");
}

int ferrite_add_rmsnorm_fwd(void* stream, const void* x, const void* r,
                            const void* w, void* h, void* y, int64_t rows,
                            int64_t dim, float eps, int dtype, int w_dtype) {
  if (int rc = check_common("add_rmsnorm_fwd", rows, dim, dtype, w_dtype)) return rc;
  if (rows == 0) return FERRITE_OK;
  if (!x || !r || !w || !h || !y)
    return fail(FERRITE_BAD_SHAPE, "add_rmsnorm_fwd: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
#define CALL(T, TW, ADD) run_fwd<T, TW, ADD>(s, x, r, w, h, y, rows, dim, eps)
  if (dtype == FERRITE_BF16 && w_dtype == FERRITE_F32) return CALL(__nv_bfloat16, float, true);
  if (dtype == FERRITE_BF16 && w_dtype == FERRITE_BF16) return CALL(__nv_bfloat16, __nv_bfloat16, true);
  if (dtype == FERRITE_F32 && w_dtype == FERRITE_F32) return CALL(float, float, true);
  if (dtype == FERRITE_F16 && w_dtype == FERRITE_F32) return CALL(__half, float, true);
#undef CALL
  return fail(FERRITE_UNSUPPORTED_DTYPE, "add_rmsnorm_fwd: dtype");
}

}  // extern "C"
