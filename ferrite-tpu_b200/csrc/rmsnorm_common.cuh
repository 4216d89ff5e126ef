// Fused residual-add + RMSNorm, forward and backward, for sm_100a: shared pieces.
//
// Memory-bound by design (0.6 FLOP/byte): the kernels stream each input once
// with 128-bit loads, keep the row in registers, reduce the row statistics in
// f32 with warp shuffles (plus a tiny shared-memory step when a row spans more
// than one warp) and write each output once.
//
// Row layout: a row of `dim` elements is split into 16-byte vectors; a "row
// group" of TPR threads owns one row and each thread holds VPT vectors of it
// (vector i*TPR + t for thread t), so global accesses of a row group are fully
// coalesced.  A CTA holds CTA/TPR row groups.
//
// Reference semantics (anxnd2211/ferrite-tpu, src/ferrite/kernels/rmsnorm.py):
//   forward  (_add_rmsnorm_kernel :52-56, _rmsnorm_kernel :46-49, _inv_rms :39-43)
//     h = x + r in f32, stored rounded; y = h * rsqrt(sum(h^2)/dim + eps) * w,
//     computed from the unrounded f32 h.
//   backward (_rmsnorm_bwd_math :159-166, _add_norm_bwd :148-153)
//     from the saved rounded h: inv, xhat = h*inv, g = dy*w,
//     dh = inv*(g - xhat*mean(g*xhat)) + dh_direct, dw = sum_rows dy*xhat.
//     Here mean(g*xhat) = inv * mean(dy*w*h), so both row sums (h^2 and dy*w*h)
//     come out of a single pass.  dw is reduced without atomics: each CTA of the
//     persistent grid writes its f32 partial row to the workspace and a second
//     kernel sums the partials in a fixed order (bitwise deterministic).
#pragma once
#include <algorithm>
#include <cstdlib>

#include "common.cuh"

namespace ferrite {
namespace norm {

template <typename T>
struct Vec {
  static constexpr int N = 16 / sizeof(T);
  __device__ __forceinline__ static void to_f(const uint4& v, float (&f)[N]) {
    const T* p = reinterpret_cast<const T*>(&v);
#pragma unroll
    for (int i = 0; i < N; ++i) f[i] = DT<T>::to_f(p[i]);
  }
  __device__ __forceinline__ static uint4 from_f(const float (&f)[N]) {
    uint4 v;
    T* p = reinterpret_cast<T*>(&v);
#pragma unroll
    for (int i = 0; i < N; ++i) p[i] = DT<T>::from_f(f[i]);
    return v;
  }
};

// Load VE consecutive weights (as f32) starting at element e.
template <typename TW, int VE>
__device__ __forceinline__ void load_w(const TW* w, int64_t e, float (&f)[VE]) {
  if constexpr (sizeof(TW) == 4) {
#pragma unroll
    for (int i = 0; i < VE; i += 4) {
      float4 v = __ldg(reinterpret_cast<const float4*>(w + e + i));
      f[i] = v.x;
      f[i + 1] = v.y;
      f[i + 2] = v.z;
      f[i + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < VE; i += 8) {
      uint4 v = ld_v4(w + e + i);
      const TW* p = reinterpret_cast<const TW*>(&v);
#pragma unroll
      for (int j = 0; j < 8 && i + j < VE; ++j) f[i + j] = DT<TW>::to_f(p[j]);
    }
  }
}

// Sum `v` (NV values) over the TPR threads of a row group.  `red` is shared
// scratch of at least (CTA/32)*NV floats; `sync` is true when TPR > 32.
template <int TPR, int NV>
__device__ __forceinline__ void row_reduce(float (&v)[NV], float* red) {
  if constexpr (TPR <= 32) {
#pragma unroll
    for (int off = TPR / 2; off > 0; off >>= 1) {
#pragma unroll
      for (int j = 0; j < NV; ++j) v[j] += __shfl_xor_sync(0xffffffffu, v[j], off);
    }
  } else {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
#pragma unroll
      for (int j = 0; j < NV; ++j) v[j] += __shfl_xor_sync(0xffffffffu, v[j], off);
    }
    constexpr int WPR = TPR / 32;  // warps per row
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
#pragma unroll
      for (int j = 0; j < NV; ++j) red[warp * NV + j] = v[j];
    }
    __syncthreads();
    const int first = (warp / WPR) * WPR;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      float s = 0.f;
#pragma unroll
      for (int q = 0; q < WPR; ++q) s += red[(first + q) * NV + j];
      v[j] = s;
    }
    __syncthreads();  // red is reused by the next row
  }
}

// ---------------------------------------------------------------------------
// launch configuration
// ---------------------------------------------------------------------------

struct Cfg {
  int vpt;  // vectors per thread (1, 2, 4, 8)
  int tpr;  // threads per row (power of two, 4..1024)
  bool vec;  // vectorised path usable
};

static int env_int(const char* name, int dflt) {
  const char* s = std::getenv(name);
  if (!s || !*s) return dflt;
  return std::atoi(s);
}

// Instantiated (vectors per thread, threads per row) pairs.  Short rows use one
// vector per thread, mid-size rows two (the default), long rows four.
static bool cfg_ok(int vpt, int tpr) {
  switch (vpt) {
    case 1: return tpr >= 4 && tpr <= 1024;
    case 2: return tpr >= 64 && tpr <= 1024;
    case 4: return tpr >= 256 && tpr <= 1024;
  }
  return false;
}

static int64_t pow2ceil(int64_t v) {
  int64_t p = 1;
  while (p < v) p <<= 1;
  return p;
}

static Cfg pick(int64_t dim, int elem, const void* const* ptrs, int nptr,
                bool bwd) {
  Cfg c{0, 0, false};
  const int ve = 16 / elem;
  if (dim % ve != 0) return c;
  for (int i = 0; i < nptr; ++i)
    if (ptrs[i] && (reinterpret_cast<uintptr_t>(ptrs[i]) & 15u)) return c;
  const int64_t nvec = dim / ve;
  int pref = bwd ? env_int("FERRITE_RMSNORM_BWD_VPT", 1) : env_int("FERRITE_RMSNORM_VPT", 2);
  if (pref != 1 && pref != 2 && pref != 4) pref = 2;
  const int order[3][3] = {{1, 2, 4}, {2, 4, 1}, {4, 2, 1}};
  const int* ord = order[pref == 1 ? 0 : (pref == 2 ? 1 : 2)];
  for (int k = 0; k < 3; ++k) {
    const int vpt = ord[k];
    const int64_t tpr = std::max<int64_t>(4, pow2ceil((nvec + vpt - 1) / vpt));
    if (tpr <= 1024 && cfg_ok(vpt, (int)tpr)) {
      c.vpt = vpt;
      c.tpr = (int)tpr;
      c.vec = true;
      return c;
    }
  }
  return c;  // row too long (or too short for the preferred shapes): scalar path
}

// Largest number of dw partial rows any plan produces: 8 per SM (the vector
// plan uses at most 4 CTAs of >= 512 threads per SM, the scalar plan one CTA of
// 8 warps per SM), and never more than the row count rounded up to 8.
static int64_t max_parts(int64_t rows, int device) {
  const int64_t r8 = ((std::max<int64_t>(rows, 1) + 7) / 8) * 8;
  return std::min<int64_t>(r8, (int64_t)num_sms(device) * 8);
}

static inline int check_common(const char* op, int64_t rows, int64_t dim, int dtype,
                        int w_dtype) {
  if (rows < 0 || dim <= 0 || dim > (1 << 24))
    return fail(FERRITE_BAD_SHAPE, "%s: bad shape rows=%lld dim=%lld", op,
                (long long)rows, (long long)dim);
  if (dtype != FERRITE_F32 && dtype != FERRITE_BF16 && dtype != FERRITE_F16)
    return fail(FERRITE_UNSUPPORTED_DTYPE, "%s: unsupported dtype %d", op, dtype);
  if (w_dtype != FERRITE_F32 && w_dtype != FERRITE_BF16)
    return fail(FERRITE_UNSUPPORTED_DTYPE, "%s: unsupported weight dtype %d", op, w_dtype);
  return injected_fault(op);
}

}  // namespace norm
}  // namespace ferrite
