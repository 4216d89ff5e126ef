// Softmax cross-entropy over f32 logit rows: the GPT loss of the reference
// (src/ferrite/model/gpt.py:147-152: log_softmax over the vocabulary, gather of
// the target's log-probability, mean over tokens) as two HBM-bound row passes.
//
//   forward : lse[r] = log sum_c exp(x[r, c])      one read of the row, with a
//             nll[r] = lse[r] - x[r, t[r]]           one-pass online max / sum
//   backward: dx[r, c] = g * (exp(x[r, c] - lse[r]) - [c == t[r]])
//             written directly in the dtype the LM-head GEMMs consume, so the
//             log-softmax backward and the f32 -> bf16 cast are one pass.
//             g = (*dloss) * scale (scale = 1 / rows for the mean), read on the
//             device so no host synchronisation is needed.
//
// One CTA per row; 16-byte loads when the row is 16-byte aligned and the
// vocabulary a multiple of 4, scalar loads otherwise.  A target outside
// [0, vocab) gives nll = NaN and no one-hot term (nothing is read out of range).
#include <cmath>
#include <type_traits>

#include "common.cuh"

namespace ferrite {
namespace xent {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

// (m, s) represents sum_i exp(x_i) = s * exp(m); merge two such partial sums.
__device__ __forceinline__ void merge(float& m, float& s, float m2, float s2) {
  const float mn = fmaxf(m, m2);
  if (mn == -INFINITY) return;  // both empty
  s = s * __expf(m - mn) + s2 * __expf(m2 - mn);
  m = mn;
}

__device__ __forceinline__ int64_t target_at(const void* t, int64_t r, int is64) {
  return is64 ? static_cast<const int64_t*>(t)[r] : (int64_t) static_cast<const int32_t*>(t)[r];
}

template <bool VEC>
__global__ void __launch_bounds__(kThreads)
    xent_fwd_kernel(const float* __restrict__ logits, const void* __restrict__ targets,
                    float* __restrict__ lse, float* __restrict__ nll, int64_t vocab, int64_t ld,
                    int is64) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float sm[kWarps], ss[kWarps];
  const int64_t r = blockIdx.x;
  const float* x = logits + r * ld;
  float m = -INFINITY, s = 0.f;
  if constexpr (VEC) {
    const int64_t nv = vocab / 4;
    for (int64_t i = threadIdx.x; i < nv; i += kThreads) {
      const uint4 u = ld_stream_v4(x + i * 4);
      const float a = __uint_as_float(u.x), b = __uint_as_float(u.y);
      const float c = __uint_as_float(u.z), d = __uint_as_float(u.w);
      const float cm = fmaxf(fmaxf(a, b), fmaxf(c, d));
      const float mn = fmaxf(m, cm);
      const float keep = m == -INFINITY ? 0.f : __expf(m - mn);
      s = s * keep + (__expf(a - mn) + __expf(b - mn)) + (__expf(c - mn) + __expf(d - mn));
      m = mn;
    }
  } else {
    for (int64_t i = threadIdx.x; i < vocab; i += kThreads) {
      const float a = x[i];
      const float mn = fmaxf(m, a);
      const float keep = m == -INFINITY ? 0.f : __expf(m - mn);
      s = s * keep + __expf(a - mn);
      m = mn;
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, off);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, off);
    merge(m, s, m2, s2);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sm[warp] = m;
    ss[warp] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = sm[0], S = ss[0];
    for (int w = 1; w < kWarps; ++w) merge(M, S, sm[w], ss[w]);
    const float l = M + logf(S);
    lse[r] = l;
    const int64_t t = target_at(targets, r, is64);
    nll[r] = (t >= 0 && t < vocab) ? l - x[t] : __int_as_float(0x7fc00000);
  }
}

template <typename TO>
__device__ __forceinline__ void store4(TO* p, float a, float b, float c, float d) {
  if constexpr (sizeof(TO) == 4) {
    *reinterpret_cast<float4*>(p) = make_float4(a, b, c, d);
  } else if constexpr (std::is_same<TO, __nv_bfloat16>::value) {
    *reinterpret_cast<uint2*>(p) = make_uint2(pack_bf16x2(a, b), pack_bf16x2(c, d));
  } else {
    *reinterpret_cast<uint2*>(p) = make_uint2(pack_f16x2(a, b), pack_f16x2(c, d));
  }
}

template <typename TO, bool VEC>
__global__ void __launch_bounds__(kThreads)
    xent_bwd_kernel(const float* __restrict__ logits, const void* __restrict__ targets,
                    const float* __restrict__ lse, const float* __restrict__ dloss, float scale,
                    TO* __restrict__ dx, int64_t vocab, int64_t ld, int64_t ld_out, int is64) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t r = blockIdx.x;
  const float* x = logits + r * ld;
  TO* o = dx + r * ld_out;
  const float g = (dloss ? *dloss : 1.0f) * scale;
  const float l = lse[r];
  const int64_t t = target_at(targets, r, is64);
  if constexpr (VEC) {
    const int64_t nv = vocab / 4;
    for (int64_t i = threadIdx.x; i < nv; i += kThreads) {
      const uint4 u = ld_stream_v4(x + i * 4);
      float v[4] = {__uint_as_float(u.x), __uint_as_float(u.y), __uint_as_float(u.z),
                    __uint_as_float(u.w)};
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = (__expf(v[j] - l) - (i * 4 + j == t ? 1.f : 0.f)) * g;
      store4<TO>(o + i * 4, v[0], v[1], v[2], v[3]);
    }
  } else {
    for (int64_t i = threadIdx.x; i < vocab; i += kThreads)
      o[i] = DT<TO>::from_f((__expf(x[i] - l) - (i == t ? 1.f : 0.f)) * g);
  }
}

static int check_args(const char* op, int64_t rows, int64_t vocab, int64_t ld, int target_dtype) {
  if (int rc = injected_fault(op)) return rc;
  if (rows < 0 || vocab <= 0 || ld < vocab)
    return fail(FERRITE_BAD_SHAPE, "%s: bad shape rows=%lld vocab=%lld ld=%lld", op,
                (long long)rows, (long long)vocab, (long long)ld);
  if (rows > 0x7fffffff) return fail(FERRITE_BAD_SHAPE, "%s: too many rows", op);
  if (target_dtype != 0 && target_dtype != 1)
    return fail(FERRITE_UNSUPPORTED_DTYPE, "%s: target dtype %d (0 = int32, 1 = int64)", op,
                target_dtype);
  return FERRITE_OK;
}

template <typename TO>
static int launch_bwd(cudaStream_t s, const float* logits, const void* targets, const float* lse,
                      const float* dloss, float scale, void* dx, int64_t rows, int64_t vocab,
                      int64_t ld, int64_t ld_out, int is64) {
  const bool vec = vocab % 4 == 0 && ld % 4 == 0 && ld_out % 4 == 0 &&
                   (reinterpret_cast<uintptr_t>(logits) & 15u) == 0 &&
                   (reinterpret_cast<uintptr_t>(dx) & (sizeof(TO) * 4 - 1)) == 0;
  if (vec)
    (void)launch_pdl(xent_bwd_kernel<TO, true>, dim3((unsigned)rows), dim3(kThreads), 0, s, logits, targets, lse, dloss, scale,
                                                                  (TO*)dx, vocab, ld, ld_out, is64);
  else
    (void)launch_pdl(xent_bwd_kernel<TO, false>, dim3((unsigned)rows), dim3(kThreads), 0, s, logits, targets, lse, dloss, scale,
                                                                   (TO*)dx, vocab, ld, ld_out, is64);
  return check_launch("xent_bwd");
}

}  // namespace xent
}  // namespace ferrite

using namespace ferrite;
using namespace ferrite::xent;

extern "C" {

int ferrite_xent_fwd(void* stream, const float* logits, const void* targets, float* lse,
                     float* nll, int64_t rows, int64_t vocab, int64_t ld, int target_dtype) {
  if (int rc = check_args("xent_fwd", rows, vocab, ld, target_dtype)) return rc;
  if (rows == 0) return FERRITE_OK;
  if (!logits || !targets || !lse || !nll) return fail(FERRITE_BAD_SHAPE, "xent_fwd: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  const bool vec = vocab % 4 == 0 && ld % 4 == 0 && (reinterpret_cast<uintptr_t>(logits) & 15u) == 0;
  if (vec)
    (void)launch_pdl(xent_fwd_kernel<true>, dim3((unsigned)rows), dim3(kThreads), 0, s, logits, targets, lse, nll, vocab, ld, target_dtype);
  else
    (void)launch_pdl(xent_fwd_kernel<false>, dim3((unsigned)rows), dim3(kThreads), 0, s, logits, targets, lse, nll, vocab, ld, target_dtype);
  return check_launch("xent_fwd");
}

int ferrite_xent_bwd(void* stream, const float* logits, const void* targets, const float* lse,
                     const float* dloss, float scale, void* dlogits, int64_t rows, int64_t vocab,
                     int64_t ld, int64_t ld_out, int target_dtype, int out_dtype) {
  if (int rc = check_args("xent_bwd", rows, vocab, ld, target_dtype)) return rc;
  if (ld_out < vocab) return fail(FERRITE_BAD_SHAPE, "xent_bwd: ld_out < vocab");
  if (rows == 0) return FERRITE_OK;
  if (!logits || !targets || !lse || !dlogits) return fail(FERRITE_BAD_SHAPE, "xent_bwd: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  if (out_dtype == FERRITE_F32)
    return launch_bwd<float>(s, logits, targets, lse, dloss, scale, dlogits, rows, vocab, ld, ld_out, target_dtype);
  if (out_dtype == FERRITE_BF16)
    return launch_bwd<__nv_bfloat16>(s, logits, targets, lse, dloss, scale, dlogits, rows, vocab, ld, ld_out, target_dtype);
  if (out_dtype == FERRITE_F16)
    return launch_bwd<__half>(s, logits, targets, lse, dloss, scale, dlogits, rows, vocab, ld, ld_out, target_dtype);
  return fail(FERRITE_UNSUPPORTED_DTYPE, "xent_bwd: output dtype %d", out_dtype);
}

}  // extern "C"
