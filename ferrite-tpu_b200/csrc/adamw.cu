// AdamW with global-norm clipping over flat f32 buffers: the reference's
// adamw_update (src/ferrite/model/train.py:59-74) as two HBM-bound passes.
//
//   pass 1  sumsq_partials_kernel: fixed grid, each CTA sums g^2 over a fixed
//           grid-stride set of 16-byte vectors -> one f32 partial per CTA;
//   pass 2  adamw_kernel: every CTA first reduces the partials in the same fixed
//           order (so all CTAs see the bitwise-same norm), then
//             g = gs * grad  (gs = 1 / ranks turns a summed all-reduce into the mean)
//             gnorm = sqrt(sum g^2), scale = min(1, clip / (gnorm + 1e-6)),
//             g' = g * scale
//             m  = b1 m + (1 - b1) g'            v = b2 v + (1 - b2) g'^2
//             p  = p - lr ((m / bc1) / (sqrt(v / bc2) + eps) + wd p)
//           with wd applied to elements [0, n_decay) only (the reference decays
//           parameters with ndim >= 2; the caller lays those out first).
// One read of g in pass 1; one read of g, m, v, p and one write of m, v, p in
// pass 2: 32 bytes per element in total.  No atomics; results are run-to-run
// deterministic.
#include <cmath>

#include "common.cuh"

namespace ferrite {
namespace adamw {

constexpr int kThreads = 256;
constexpr int kMaxPartials = 1024;

__device__ __forceinline__ float block_sum(float v, float* sm) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) sm[warp] = v;
  __syncthreads();
  float t = 0.f;
  if (threadIdx.x == 0)
    for (int w = 0; w < kThreads / 32; ++w) t += sm[w];
  return t;  // valid in thread 0
}

__global__ void __launch_bounds__(kThreads)
    sumsq_partials_kernel(const float* __restrict__ g, int64_t n, float gs, float* __restrict__ partials) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float sm[kThreads / 32];
  const int64_t nv = n / 4;
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  float acc = 0.f;
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < nv; i += stride) {
    const float4 x = __ldcs(reinterpret_cast<const float4*>(g) + i);
    acc = fmaf(x.x, x.x, acc);
    acc = fmaf(x.y, x.y, acc);
    acc = fmaf(x.z, x.z, acc);
    acc = fmaf(x.w, x.w, acc);
  }
  if (blockIdx.x == 0)  // the scalar tail (n % 4 elements)
    for (int64_t i = nv * 4 + threadIdx.x; i < n; i += kThreads) acc = fmaf(g[i], g[i], acc);
  const float t = block_sum(acc, sm);
  if (threadIdx.x == 0) partials[blockIdx.x] = t * gs * gs;
}

struct Hyper {
  float lr, b1, b2, eps, wd, bc1, bc2, clip, gs;  // gs: gradient pre-scale (1 / ranks for a summed all-reduce)
};

__device__ __forceinline__ void update1(float& p, float g, float& m, float& v, float scale,
                                        const Hyper& h, bool decay) {
  const float gc = (g * h.gs) * scale;
  m = h.b1 * m + (1.f - h.b1) * gc;
  v = h.b2 * v + (1.f - h.b2) * gc * gc;
  float u = (m / h.bc1) / (sqrtf(v / h.bc2) + h.eps);
  if (decay) u += h.wd * p;
  p = p - h.lr * u;
}

__global__ void __launch_bounds__(kThreads)
    adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                 float* __restrict__ v, int64_t n, int64_t n_decay, const float* __restrict__ partials,
                 int n_partials, Hyper h, float* __restrict__ gnorm_out) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float sm[kThreads / 32];
  __shared__ float s_scale;
  // identical fixed-order reduction of the partials in every CTA
  float acc = 0.f;
  for (int i = threadIdx.x; i < n_partials; i += kThreads) acc += partials[i];
  const float total = block_sum(acc, sm);
  if (threadIdx.x == 0) {
    const float gnorm = sqrtf(total);
    s_scale = fminf(1.0f, h.clip / (gnorm + 1e-6f));
    if (blockIdx.x == 0 && gnorm_out) *gnorm_out = gnorm;
  }
  __syncthreads();
  const float scale = s_scale;
  const int64_t nv = n / 4;
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < nv; i += stride) {
    float4 pp = reinterpret_cast<float4*>(p)[i];
    const float4 gg = __ldcs(reinterpret_cast<const float4*>(g) + i);
    float4 mm = reinterpret_cast<float4*>(m)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
    const int64_t e = i * 4;
    update1(pp.x, gg.x, mm.x, vv.x, scale, h, e + 0 < n_decay);
    update1(pp.y, gg.y, mm.y, vv.y, scale, h, e + 1 < n_decay);
    update1(pp.z, gg.z, mm.z, vv.z, scale, h, e + 2 < n_decay);
    update1(pp.w, gg.w, mm.w, vv.w, scale, h, e + 3 < n_decay);
    reinterpret_cast<float4*>(p)[i] = pp;
    reinterpret_cast<float4*>(m)[i] = mm;
    reinterpret_cast<float4*>(v)[i] = vv;
  }
  if (blockIdx.x == 0)
    for (int64_t i = nv * 4 + threadIdx.x; i < n; i += kThreads) update1(p[i], g[i], m[i], v[i], scale, h, i < n_decay);
}

static int n_partials_for(int64_t n) {
  const int64_t want = (n / 4 + kThreads * 8 - 1) / (kThreads * 8);  // ~8 vectors per thread
  return (int)std::max<int64_t>(1, std::min<int64_t>(kMaxPartials, want));
}

}  // namespace adamw
}  // namespace ferrite

using namespace ferrite;
using namespace ferrite::adamw;

extern "C" {

size_t ferrite_adamw_workspace_size(int64_t n) {
  return n <= 0 ? 0 : (size_t)n_partials_for(n) * sizeof(float);
}

int ferrite_adamw_step(void* stream, float* params, const float* grads, float* m, float* v,
                       int64_t n, int64_t n_decay, float lr, float b1, float b2, float eps,
                       float weight_decay, int64_t step, float clip, float grad_scale,
                       float* gnorm_out, void* workspace, size_t workspace_bytes) {
  if (int rc = injected_fault("adamw_step")) return rc;
  if (n < 0 || n_decay < 0 || n_decay > n) return fail(FERRITE_BAD_SHAPE, "adamw_step: n=%lld n_decay=%lld", (long long)n, (long long)n_decay);
  if (step < 1) return fail(FERRITE_BAD_SHAPE, "adamw_step: step must be >= 1 (got %lld)", (long long)step);
  if (n == 0) return FERRITE_OK;
  if (!params || !grads || !m || !v || !workspace) return fail(FERRITE_BAD_SHAPE, "adamw_step: null pointer");
  const int np = n_partials_for(n);
  if (workspace_bytes < (size_t)np * sizeof(float))
    return fail(FERRITE_WORKSPACE_TOO_SMALL, "adamw_step: workspace %zu < %zu bytes", workspace_bytes,
                (size_t)np * sizeof(float));
  for (const void* ptr : {(const void*)params, (const void*)grads, (const void*)m, (const void*)v})
    if (reinterpret_cast<uintptr_t>(ptr) & 15u)
      return fail(FERRITE_BAD_ALIGNMENT, "adamw_step: buffers must be 16-byte aligned");
  cudaStream_t s = (cudaStream_t)stream;
  float* partials = static_cast<float*>(workspace);
  (void)launch_pdl(sumsq_partials_kernel, dim3(np), dim3(kThreads), 0, s, grads, n, grad_scale, partials);
  if (int rc = check_launch("adamw_sumsq")) return rc;
  Hyper h;
  h.lr = lr;
  h.b1 = b1;
  h.b2 = b2;
  h.eps = eps;
  h.wd = weight_decay;
  h.bc1 = (float)(1.0 - std::pow((double)b1, (double)step));
  h.bc2 = (float)(1.0 - std::pow((double)b2, (double)step));
  h.clip = clip;
  h.gs = grad_scale;
  const int grid = std::min<int64_t>((n / 4 + kThreads - 1) / kThreads + 1, (int64_t)num_sms(current_device()) * 8);
  (void)launch_pdl(adamw_kernel, dim3(grid), dim3(kThreads), 0, s, params, grads, m, v, n, n_decay, partials, np, h, gnorm_out);
  return check_launch("adamw_update");
}

}  // extern "C"
