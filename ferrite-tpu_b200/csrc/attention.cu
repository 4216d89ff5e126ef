// Causal flash attention for sm_100a: forward, delta prep, dK/dV and dQ.
//
// Tensor-core path (bf16/f16, head_dim 64 or 128, sk a multiple of 128), all
// warp-specialised with TMA loads, tcgen05.mma into TMEM and bounded mbarrier waits:
//   forward (attn_fwd_tc_kernel): a CTA holds two 128-row query tiles (d = 128) whose
//     softmax warpgroups ping-pong on one tensor core, or one tile (d = 64, two CTAs
//     per SM).  S = Q K^T lands in TMEM; the softmax writes P back into TMEM as packed
//     pairs (into S's own columns, or at d = 64 into free columns so the next S need
//     not wait for P V); O accumulates in TMEM through TS-form MMAs and is rescaled
//     only when the running max grows by more than 2^8.  Fully masked causal tiles
//     are never loaded.
//   delta prep (bwd_prep_vec_kernel): rowsum(dO * O), vectorised.
//   backward, two kernels: dK/dV per (128-key tile, slice) CTA over 128-query tiles
//     (attn_dkv_wide_kernel), writing the rounded dS to a scratch slot; then dQ as a
//     tensor-core GEMM over that dS (attn_dq_ds_kernel).
//   backward, fused (attn_bwd_fused_kernel, from 4096 queries on): the same dK/dV work
//     and the dQ-from-dS work as units of one persistent launch, dS read back from L2
//     as soon as a query-tile pair is complete, with a scheduler warp claiming units.
// The sections below describe each kernel in detail.
//
// Reference numerics (src/ferrite/kernels/flash_attention.py): scores
// scale * q k^T in f32 (:103-105), finite MASK_VALUE on the causal diagonal
// tile (:44, :80-83), online softmax with f32 statistics (:108-115), P rounded
// to v.dtype before P V (:114), normalise once after the last key block and
// lse = m + log l (:122-127).  Exponentials are evaluated as exp2 of
// log2(e)-prescaled scores (the same function up to f32 rounding).
//
// Everything else (f32 inputs, other head dims, ragged sequence lengths) runs
// a CUDA-core path with the same blockwise semantics: one warp per query (or
// key) row, blocks of 32 keys (queries).
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <type_traits>

#include "common.cuh"

namespace ferrite {
FERRITE_DEFINE_STATUS_READER(status_attention)

namespace attn {

constexpr float kMaskValue = -0.7f * 3.40282346638528859812e+38f;  // -0.7 * FLT_MAX
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// Element strides (batch, head, sequence) of a [b, h, s, d] operand whose d is
// unit-stride, and the head count that splits the flattened batch*head index.
// Contiguous [b, h, s, d] is {h*s*d, s*d, d}; the GPT block's packed
// [b, s, 3, h, d] projection read in place is {3*h*s*d, d, 3*h*d} per slot.
struct Bhsd {
  int64_t b, h, s;
  int nh;
  __host__ __device__ __forceinline__ int64_t row(int64_t bh, int64_t r) const {
    return (bh / nh) * b + (bh % nh) * h + r * s;
  }
};

// ===========================================================================
// delta = rowsum(dO * O) (flash_attention.py:328)
// ===========================================================================

template <typename T>
__global__ void __launch_bounds__(256)
    bwd_prep_kernel(const T* __restrict__ dout, const T* __restrict__ out,
                    float* __restrict__ delta, Bhsd ld, Bhsd lo, int64_t rows, int s_len, int d) {
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int64_t bh = row / s_len, r = row % s_len;
  const T* a = dout + ld.row(bh, r);
  const T* b = out + lo.row(bh, r);
  float s = 0.f;
  for (int j = lane; j < d; j += 32) s = fmaf(DT<T>::to_f(a[j]), DT<T>::to_f(b[j]), s);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (lane == 0) delta[row] = s;
}

// Vectorised delta: CTA (x, bh) covers prep_rows_per_cta(VPR) sequence rows of
// slice bh; a row is read as VPR 16-byte vectors by VPR adjacent lanes (VPR =
// d / (16 / sizeof(T)), a power of two <= 32) and reduced with xor shuffles
// inside that lane group.  No integer division on the hot path.
__host__ __device__ constexpr int prep_rows_per_cta(int vpr) {
  return 256 / vpr > 128 ? 256 / vpr : 128;  // at least one full pass of 256 threads
}

template <typename T, int VPR>
__global__ void __launch_bounds__(256)
    bwd_prep_vec_kernel(const T* __restrict__ dout, const T* __restrict__ out,
                        float* __restrict__ delta, Bhsd ld, Bhsd lo, int s_len) {
  pdl_launch_dependents();
  pdl_wait();
  constexpr int kElems = 16 / sizeof(T);
  constexpr int kRowsPerPass = 256 / VPR;
  constexpr int kPasses = prep_rows_per_cta(VPR) / kRowsPerPass;
  const int bh = blockIdx.y;
  const int sub = threadIdx.x % VPR, rloc = threadIdx.x / VPR;
  const T* db = dout + ld.row(bh, 0) + sub * kElems;
  const T* ob = out + lo.row(bh, 0) + sub * kElems;
  const int r_begin = blockIdx.x * prep_rows_per_cta(VPR);
#pragma unroll 2
  for (int pass = 0; pass < kPasses; ++pass) {
    const int r = r_begin + pass * kRowsPerPass + rloc;
    float acc = 0.f;
    if (r < s_len) {
      const uint4 a = ld_stream_v4(db + (int64_t)r * ld.s);
      const uint4 b = ld_stream_v4(ob + (int64_t)r * lo.s);
      const T* ea = reinterpret_cast<const T*>(&a);
      const T* eb = reinterpret_cast<const T*>(&b);
#pragma unroll
      for (int e = 0; e < kElems; ++e) acc = fmaf(DT<T>::to_f(ea[e]), DT<T>::to_f(eb[e]), acc);
    }
#pragma unroll
    for (int off = VPR / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (sub == 0 && r < s_len) delta[(int64_t)bh * s_len + r] = acc;
  }
}

// ===========================================================================
// CUDA-core path (any dtype, head_dim <= 256)
// ===========================================================================

constexpr int kSimtMaxD = 256;
constexpr int kSimtWarps = 4;  // rows per CTA

template <typename T>
__device__ __forceinline__ float round_to(float v) {
  return DT<T>::to_f(DT<T>::from_f(v));
}

// Forward: one warp per query row; keys in blocks of 32 (lane j owns key j of
// the block for the scores, and d/32 output dims for the accumulator).
template <typename T>
__global__ void __launch_bounds__(kSimtWarps * 32)
    simt_fwd_kernel(const T* __restrict__ q, const T* __restrict__ k,
                    const T* __restrict__ v, T* __restrict__ o, float* __restrict__ lse,
                    Bhsd lq, Bhsd lk, Bhsd lv, Bhsd lo, int sq, int sk, int d, float scale,
                    int causal) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float qs[kSimtWarps][kSimtMaxD];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t bh = blockIdx.y;
  const int row = blockIdx.x * kSimtWarps + warp;
  const bool active = row < sq;
  const T* qr = q + lq.row(bh, active ? row : 0);
  const T* kb = k + lk.row(bh, 0);
  const T* vb = v + lv.row(bh, 0);
  for (int j = lane; j < d; j += 32) qs[warp][j] = DT<T>::to_f(qr[j]);
  __syncwarp();
  constexpr int DPL = kSimtMaxD / 32;  // output dims per lane (max)
  float acc[DPL];
#pragma unroll
  for (int i = 0; i < DPL; ++i) acc[i] = 0.f;
  float m = -INFINITY, l = 0.f;
  const int kend = causal ? min(sk, row + 1 + (sk - sq)) : sk;
  for (int k0 = 0; active && k0 < kend; k0 += 32) {
    const int key = k0 + lane;
    float s = kMaskValue;
    if (key < sk) {
      const T* kr = kb + (int64_t)key * lk.s;
      float dot = 0.f;
      for (int j = 0; j < d; ++j) dot = fmaf(qs[warp][j], DT<T>::to_f(kr[j]), dot);
      s = dot * scale;
      if (causal && key > row + (sk - sq)) s = kMaskValue;
    }
    float bm = s;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, off));
    const float m_new = fmaxf(m, bm);
    float p = (key < sk) ? expf(s - m_new) : 0.f;
    const float alpha = expf(m - m_new);
    float ps = p;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
    l = alpha * l + ps;
    m = m_new;
    const float pr = round_to<T>(p);
#pragma unroll
    for (int i = 0; i < DPL; ++i) acc[i] *= alpha;
    for (int jj = 0; jj < 32; ++jj) {
      const float pj = __shfl_sync(0xffffffffu, pr, jj);
      const int kk = k0 + jj;
      if (kk >= sk) break;
      const T* vr = vb + (int64_t)kk * lv.s;
#pragma unroll
      for (int i = 0; i < DPL; ++i) {
        const int dd = lane + 32 * i;
        if (dd < d) acc[i] = fmaf(pj, DT<T>::to_f(vr[dd]), acc[i]);
      }
    }
  }
  if (!active) return;
  const float inv = 1.0f / l;
  T* orow = o + lo.row(bh, row);
#pragma unroll
  for (int i = 0; i < DPL; ++i) {
    const int dd = lane + 32 * i;
    if (dd < d) orow[dd] = DT<T>::from_f(acc[i] * inv);
  }
  if (lane == 0) lse[bh * sq + row] = m + logf(l);
}

// dQ: one warp per query row, keys in blocks of 32.
template <typename T>
__global__ void __launch_bounds__(kSimtWarps * 32)
    simt_bwd_dq_kernel(const T* __restrict__ q, const T* __restrict__ k,
                       const T* __restrict__ v, const T* __restrict__ dout,
                       const float* __restrict__ lse, const float* __restrict__ delta,
                       T* __restrict__ dq, Bhsd lq, Bhsd lk, Bhsd lv, Bhsd ldo, Bhsd ldq,
                       int sq, int sk, int d, float scale, int causal) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float qs[kSimtWarps][kSimtMaxD];
  __shared__ float ds_[kSimtWarps][kSimtMaxD];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t bh = blockIdx.y;
  const int row = blockIdx.x * kSimtWarps + warp;
  if (row >= sq) return;
  const T* qr = q + lq.row(bh, row);
  const T* dor = dout + ldo.row(bh, row);
  for (int j = lane; j < d; j += 32) {
    qs[warp][j] = DT<T>::to_f(qr[j]);
    ds_[warp][j] = DT<T>::to_f(dor[j]);
  }
  __syncwarp();
  const float lr = lse[bh * sq + row], dl = delta[bh * sq + row];
  const T* kb = k + lk.row(bh, 0);
  const T* vb = v + lv.row(bh, 0);
  constexpr int DPL = kSimtMaxD / 32;
  float acc[DPL];
#pragma unroll
  for (int i = 0; i < DPL; ++i) acc[i] = 0.f;
  const int kend = causal ? min(sk, row + 1 + (sk - sq)) : sk;
  for (int k0 = 0; k0 < kend; k0 += 32) {
    const int key = k0 + lane;
    float dsv = 0.f;
    if (key < sk) {
      const T* kr = kb + (int64_t)key * lk.s;
      const T* vr = vb + (int64_t)key * lv.s;
      float sdot = 0.f, pdot = 0.f;
      for (int j = 0; j < d; ++j) {
        sdot = fmaf(qs[warp][j], DT<T>::to_f(kr[j]), sdot);
        pdot = fmaf(ds_[warp][j], DT<T>::to_f(vr[j]), pdot);
      }
      float s = sdot * scale;
      if (causal && key > row + (sk - sq)) s = kMaskValue;
      const float p = expf(s - lr);
      dsv = round_to<T>(p * (pdot - dl));
    }
    for (int jj = 0; jj < 32; ++jj) {
      const float dj = __shfl_sync(0xffffffffu, dsv, jj);
      const int kk = k0 + jj;
      if (kk >= sk) break;
      const T* kr = kb + (int64_t)kk * lk.s;
#pragma unroll
      for (int i = 0; i < DPL; ++i) {
        const int dd = lane + 32 * i;
        if (dd < d) acc[i] = fmaf(dj, DT<T>::to_f(kr[dd]), acc[i]);
      }
    }
  }
  T* out = dq + ldq.row(bh, row);
#pragma unroll
  for (int i = 0; i < DPL; ++i) {
    const int dd = lane + 32 * i;
    if (dd < d) out[dd] = DT<T>::from_f(acc[i] * scale);
  }
}

// dK, dV: one warp per key row, queries in blocks of 32.
template <typename T>
__global__ void __launch_bounds__(kSimtWarps * 32)
    simt_bwd_dkv_kernel(const T* __restrict__ q, const T* __restrict__ k,
                        const T* __restrict__ v, const T* __restrict__ dout,
                        const float* __restrict__ lse, const float* __restrict__ delta,
                        T* __restrict__ dk, T* __restrict__ dv, Bhsd lq, Bhsd lk, Bhsd lv,
                        Bhsd ldo, Bhsd ldk, Bhsd ldv, int sq, int sk, int d, float scale,
                        int causal) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float ks[kSimtWarps][kSimtMaxD];
  __shared__ float vs[kSimtWarps][kSimtMaxD];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t bh = blockIdx.y;
  const int key = blockIdx.x * kSimtWarps + warp;
  if (key >= sk) return;
  const T* kr = k + lk.row(bh, key);
  const T* vr = v + lv.row(bh, key);
  for (int j = lane; j < d; j += 32) {
    ks[warp][j] = DT<T>::to_f(kr[j]);
    vs[warp][j] = DT<T>::to_f(vr[j]);
  }
  __syncwarp();
  const T* qb = q + lq.row(bh, 0);
  const T* db = dout + ldo.row(bh, 0);
  constexpr int DPL = kSimtMaxD / 32;
  float ak[DPL], av[DPL];
#pragma unroll
  for (int i = 0; i < DPL; ++i) ak[i] = av[i] = 0.f;
  const int qstart = causal ? max(0, key - (sk - sq)) : 0;
  for (int q0 = qstart - (qstart % 32); q0 < sq; q0 += 32) {
    const int qi = q0 + lane;
    float pv = 0.f, dsv = 0.f;
    if (qi < sq && qi >= qstart) {
      const T* qr = qb + (int64_t)qi * lq.s;
      const T* dr = db + (int64_t)qi * ldo.s;
      float sdot = 0.f, pdot = 0.f;
      for (int j = 0; j < d; ++j) {
        sdot = fmaf(DT<T>::to_f(qr[j]), ks[warp][j], sdot);
        pdot = fmaf(DT<T>::to_f(dr[j]), vs[warp][j], pdot);
      }
      float s = sdot * scale;
      if (causal && key > qi + (sk - sq)) s = kMaskValue;
      const float p = expf(s - lse[bh * sq + qi]);
      pv = round_to<T>(p);
      dsv = round_to<T>(p * (pdot - delta[bh * sq + qi]));
    }
    for (int jj = 0; jj < 32; ++jj) {
      const float pj = __shfl_sync(0xffffffffu, pv, jj);
      const float dj = __shfl_sync(0xffffffffu, dsv, jj);
      const int qq = q0 + jj;
      if (qq >= sq) break;
      const T* qr = qb + (int64_t)qq * lq.s;
      const T* dr = db + (int64_t)qq * ldo.s;
#pragma unroll
      for (int i = 0; i < DPL; ++i) {
        const int dd = lane + 32 * i;
        if (dd < d) {
          av[i] = fmaf(pj, DT<T>::to_f(dr[dd]), av[i]);
          ak[i] = fmaf(dj, DT<T>::to_f(qr[dd]), ak[i]);
        }
      }
    }
  }
  T* okr = dk + ldk.row(bh, key);
  T* ovr = dv + ldv.row(bh, key);
#pragma unroll
  for (int i = 0; i < DPL; ++i) {
    const int dd = lane + 32 * i;
    if (dd < d) {
      okr[dd] = DT<T>::from_f(ak[i] * scale);
      ovr[dd] = DT<T>::from_f(av[i]);
    }
  }
}

// ===========================================================================
// Tensor-core forward
// ===========================================================================
//
// One CTA = 256 query rows (two 128-row tiles Q0, Q1) of one (batch, head):
//   warp 0       TMA: Q0, Q1 once; K/V tiles into a 2-slot ring.  Causal: only
//                the KV tiles up to the block's diagonal are ever loaded.
//   warp 1       MMA issuer (one lane), ping-pong over the two query tiles:
//                  S_g = Q_g K_j^T                    (SS, f32 in TMEM)
//                  O_g += P_g V_j                     (TS: P_g read from TMEM)
//                in the order S0(0) S1(0) | PV0(j) S0(j+1) PV1(j) S1(j+1) | ...,
//                so one group's softmax overlaps the other group's MMAs.
//   warps 4-7    softmax group 0 (rows of Q0), warps 8-11 group 1 (Q1); one
//                thread per row / TMEM lane.  Each tile: load the S row (128
//                columns) into registers, row max in the log2 domain, and
//                  p = 2^(s * scale * log2e - m)
//                rounded to the input dtype and written back into the first 64
//                S columns as packed pairs (the A operand of the next PV MMA).  O lives in TMEM: it is rescaled (ld, multiply, st)
//                only when the running max grows by more than 2^8, otherwise p
//                keeps using the stale max (l and O share it, so O / l is
//                unchanged up to rounding).  After the last tile O / l is stored
//                and lse = (m + log2 l) * ln 2.
// TMEM: S0 [0,128), S1 [128,256), O0 [256, 256+D), O1 [256+D, 256+2D);
// with one query tile per CTA (NG = 1): S0 [0,128), O0 [128, 128+D).
// MMAs issued by one thread execute in issue order, so S_g(j+1) (which
// overwrites the P_g(j) columns) is issued only after PV_g(j).

constexpr int TQ = 128;  // query rows per tile (TMEM lanes)
constexpr int TK = 128;  // keys per KV tile
constexpr float kRescaleLog2 = 8.0f;

// NG: query tiles (softmax groups) per CTA.  NG = 2 ping-pongs two groups on one
// tensor core; NG = 1 (d = 64) uses 256 TMEM columns and ~81 KB of shared memory,
// so two CTAs share an SM and overlap each other's set-up and epilogue -- what
// dominates at short sequence lengths.
template <int D, int NG = 2>
struct FwdSmem {
  static constexpr int kChunks = D / 64;      // 128-byte swizzle chunks along d
  static constexpr int kQBytes = TQ * D * 2;  // one Q tile (K-major)
  static constexpr int kKBytes = TK * D * 2;  // K tile (K-major)
  static constexpr int kVBytes = TK * D * 2;  // V tile (MN-major for the B operand)
  static constexpr int kStageBytes = kKBytes + kVBytes;
  static constexpr int kQOff = 0;  // Q0 (, Q1)
  static constexpr int kKVOff = NG * kQBytes;
  static constexpr int kBarOff = kKVOff + 2 * kStageBytes;
  // q_full, k_full[2], v_full[2], k_empty[2], v_empty[2], s_full[2], p_full[2], pv_done[2],
  // p_half[2], s_free[2]
  static constexpr int kNumBars = 19;
  static constexpr int kTotal = 1024 + kBarOff + kNumBars * 8 + 16;
};

struct FwdParams {
  int sq, sk;
  float scale_log2;  // scale * log2(e)
  int causal;
  void* o;
  Bhsd lo;     // output layout
  float* lse;  // [b*h, sq]
  int nq_blocks;  // query blocks of NG * 128 rows
};

// Byte offset of 16-byte granule `col_granule` of row `row` in a [rows x 64]
// 16-bit K-major tile stored with the 128-byte swizzle (granule ^= row % 8).
__device__ __forceinline__ uint32_t swz128(int row, int col_granule) {
  return (uint32_t)(row * 128 + ((col_granule ^ (row & 7)) << 4));
}

// CTA order of the causal tensor-core kernels.  The grid is (tiles, slices); the
// linear CTA index is mapped to (tile, slice) in batches of kOrderBatch slices with
// the tile index running slowest inside a batch.  The callers number tiles heaviest
// first, so a batch's heavy CTAs start before its light ones and the grid ends on
// light CTAs (a plain (tile, slice) grid ended on the last slice's heaviest tile);
// a batch's few slices keep the tiles they share in L2.
// Short sequences (fewer than 16 tiles a slice) keep the plain order, which measured
// 4% faster there.
constexpr int kOrderBatch = 8;
__device__ __forceinline__ void batched_order(int ntiles, int nslices, int& tile, int& slice) {
  if (ntiles < 16) {
    tile = (int)blockIdx.x;
    slice = (int)blockIdx.y;
    return;
  }
  const int lin = (int)blockIdx.x + (int)blockIdx.y * (int)gridDim.x;
  const int per_batch = kOrderBatch * ntiles;
  const int batch = lin / per_batch;
  const int s0 = batch * kOrderBatch;
  const int nb = min(kOrderBatch, nslices - s0);
  const int idx = lin - batch * per_batch;
  tile = idx / nb;
  slice = s0 + idx % nb;
}

// Warps: 0 TMA producer, 1 MMA issuer, then 4 softmax warps per query tile (the
// first at warp kSoftWarp0; a softmax warp reads TMEM lanes 32 * (warp % 4) on).
// NG = 1 has no idle warps, so 192 threads x 2 CTAs leave 168 registers a thread.
template <int NG>
constexpr int fwd_soft_warp0() { return NG == 1 ? 2 : 4; }
template <int NG>
constexpr int fwd_threads() { return 32 * (fwd_soft_warp0<NG>() + 4 * NG); }
template <int NG>
constexpr int fwd_tmem_cols() { return NG == 2 ? 512 : 256; }

template <int D, bool BF16, int NG>
__global__ void __launch_bounds__(fwd_threads<NG>(), NG == 1 ? 2 : 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tq,
                       const __grid_constant__ CUtensorMap tk,
                       const __grid_constant__ CUtensorMap tv, const FwdParams p) {
  using L = FwdSmem<D, NG>;
  constexpr uint32_t kOCol = NG * 128;  // O_g at kOCol + g * D (S_g at g * 128)
  // One query tile at d = 64 leaves TMEM columns [192, 256) free: P goes there instead of
  // into S's own columns, so S(j + 1) is issued as soon as the softmax has read S(j)
  // rather than after P V(j) -- the softmax of tile j + 1 no longer waits for S.
  constexpr bool kSepP = NG == 1 && 128 + D + 64 <= fwd_tmem_cols<NG>();
  constexpr uint32_t kPCol = 128 + D;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* q_full = bars + 0;
  // K and V tiles have separate barriers: K_j is released as soon as both S_g(j)
  // products are done, well before P V_j, so K_{j+2} streams in a full softmax
  // period earlier than a combined K/V slot would allow.
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = bars + 3;
  uint64_t* k_empty = bars + 5;
  uint64_t* v_empty = bars + 7;
  uint64_t* s_full = bars + 9;
  uint64_t* p_full = bars + 11;
  uint64_t* pv_done = bars + 13;
  // P columns of keys [0, 64) written: the first half of P V may start
  uint64_t* p_half = bars + 15;
  // kSepP: the softmax has read all of S (the next S may overwrite it)
  uint64_t* s_free = bars + 17;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::kNumBars);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Heaviest (last) query blocks first: causal work grows with the index.
  int qtile, bh;
  batched_order(p.nq_blocks, (int)gridDim.y, qtile, bh);
  const int qb = p.nq_blocks - 1 - qtile;  // heaviest (last) query blocks first
  const int hh = bh % p.lo.nh, bb = bh / p.lo.nh;  // TMA coordinates of the slice
  const int q0 = qb * NG * TQ;
  const int diag_shift = p.sk - p.sq;  // causal: key <= query + diag_shift
  int n_kv = (p.sk + TK - 1) / TK;
  if (p.causal) {
    const int last_key = min(p.sk - 1, q0 + NG * TQ - 1 + diag_shift);
    n_kv = last_key < 0 ? 0 : last_key / TK + 1;
  }

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);  // one arrival per softmax warp of the group
      mbar_init(&p_half[i], 4);
      mbar_init(&pv_done[i], 1);
      mbar_init(&s_free[i], 4);
    }
    *abort = 0;
    fence_mbar_init();
    // The first loads (Q0, Q1, K0, K1, V0: every slot is still free) are issued
    // before the TMEM allocation below, which waits for the SM's previous CTA to
    // release its columns: the tiles then stream in under that CTA's tail.
    if (n_kv > 0) {
      tma_prefetch_desc(&tq);
      tma_prefetch_desc(&tk);
      tma_prefetch_desc(&tv);
      pdl_wait();  // q, k, v may come from the previous kernel in the stream
      mbar_arrive_expect_tx(q_full, NG * L::kQBytes);
#pragma unroll
      for (int g = 0; g < NG; ++g)
#pragma unroll
        for (int c = 0; c < L::kChunks; ++c)
          tma_load_4d(smem + L::kQOff + g * L::kQBytes + c * (TQ * 128), &tq, q_full, c * 64,
                      q0 + g * TQ, hh, bb);
      for (int i = 0; i < 2 && i < n_kv; ++i) {
        uint8_t* sk_ = smem + L::kKVOff + i * L::kStageBytes;
        mbar_arrive_expect_tx(&k_full[i], L::kKBytes);
#pragma unroll
        for (int c = 0; c < L::kChunks; ++c)
          tma_load_4d(sk_ + c * (TK * 128), &tk, &k_full[i], c * 64, i * TK, hh, bb);
      }
      uint8_t* sv0 = smem + L::kKVOff + L::kKBytes;
      mbar_arrive_expect_tx(&v_full[0], L::kVBytes);
#pragma unroll
      for (int c = 0; c < L::kChunks; ++c)
        tma_load_4d(sv0 + c * (TK * 128), &tv, &v_full[0], c * 64, 0, hh, bb);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, fwd_tmem_cols<NG>());
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_launch_dependents();  // every CTA holds its TMEM before the next kernel is scheduled
  pdl_wait();
  if (warp == 0) {
    if (lane == 0 && n_kv > 0) {
      // K runs one tile ahead of V: K0, K1, V0 (issued above), K2, V1, K3, V2, ...
      for (int i = 2; i <= n_kv; ++i) {
        if (i < n_kv) {
          const int s = i & 1;
          if (!mbar_wait(&k_empty[s], ((i >> 1) & 1) ^ 1, abort, 10)) break;
          uint8_t* sk_ = smem + L::kKVOff + s * L::kStageBytes;
          mbar_arrive_expect_tx(&k_full[s], L::kKBytes);
#pragma unroll
          for (int c = 0; c < L::kChunks; ++c)
            tma_load_4d(sk_ + c * (TK * 128), &tk, &k_full[s], c * 64, i * TK, hh, bb);
        }
        if (i >= 1) {
          const int j = i - 1, s = j & 1;
          if (!mbar_wait(&v_empty[s], ((j >> 1) & 1) ^ 1, abort, 19)) break;
          uint8_t* sv_ = smem + L::kKVOff + s * L::kStageBytes + L::kKBytes;
          mbar_arrive_expect_tx(&v_full[s], L::kVBytes);
#pragma unroll
          for (int c = 0; c < L::kChunks; ++c)
            tma_load_4d(sv_ + c * (TK * 128), &tv, &v_full[s], c * 64, j * TK, hh, bb);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && n_kv > 0) {
      constexpr uint32_t idesc_s = make_idesc_f16(TQ, TK, BF16, false, false);
      constexpr uint32_t idesc_o = make_idesc_f16(TQ, D, BF16, false, true);
      const uint32_t sq_ = smem_u32(smem + L::kQOff);
      bool ok = mbar_wait(q_full, 0, abort, 11) && mbar_wait(&k_full[0], 0, abort, 12);
      // Descriptors are built once; each MMA adds a compile-time byte offset.
      const uint64_t dq_base = make_sdesc(sq_, 16, 1024);
      const uint64_t dk_base = make_sdesc(smem_u32(smem + L::kKVOff), 16, 1024);
      const uint64_t dv_base = make_sdesc(smem_u32(smem + L::kKVOff + L::kKBytes), TK * 128, 1024);
      auto issue_s = [&](int g, int j) {
        const uint64_t dq = sdesc_at(dq_base, g * L::kQBytes);
        const uint64_t dk = sdesc_at(dk_base, (j & 1) * L::kStageBytes);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t qo = (kk >> 2) * (TQ * 128) + (kk & 3) * 32;
          const uint32_t ko = (kk >> 2) * (TK * 128) + (kk & 3) * 32;
          tc_mma_f16_ss(tmem + g * 128, sdesc_at(dq, qo), sdesc_at(dk, ko), idesc_s, kk != 0);
        }
        tc_commit(&s_full[g]);
      };
      // O_g += P_g V_j over keys [64 hh, 64 hh + 64): the first half is issued as
      // soon as the softmax has written that half of P (p_half), the second with S
      // of the next tile, so the group's next S waits for half a P V, not a whole one.
      auto issue_pv = [&](int g, int j, int hh) {
        const uint64_t dv = sdesc_at(dv_base, (j & 1) * L::kStageBytes);
        const uint32_t pa = tmem + (kSepP ? kPCol : g * 128);  // P_g: packed pairs (S columns [0, 64) or kPCol)
#pragma unroll
        for (int kk = hh * 4; kk < hh * 4 + 4; ++kk)
          tc_mma_f16_ts(tmem + kOCol + g * D, pa + kk * 8, sdesc_at(dv, kk * 2048), idesc_o,
                        (j > 0 || kk > 0) ? 1u : 0u);
        if (hh == 1) tc_commit(&pv_done[g]);
      };
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        if constexpr (NG == 2) issue_s(1, 0);
        tc_commit(&k_empty[0]);  // K_0 no longer read once both S_g(0) complete
      }
      if constexpr (NG == 1) {
        for (int j = 0; ok && j < n_kv; ++j) {
          if (!mbar_wait(&p_half[0], j & 1, abort, 12)) break;
          if (!mbar_wait(&v_full[j & 1], (j >> 1) & 1, abort, 18)) break;
          tc_fence_after();
          issue_pv(0, j, 0);
          if constexpr (kSepP) {
            if (j + 1 < n_kv) {
              if (!mbar_wait(&s_free[0], j & 1, abort, 20)) break;
              if (!mbar_wait(&k_full[(j + 1) & 1], ((j + 1) >> 1) & 1, abort, 14)) break;
              tc_fence_after();
              issue_s(0, j + 1);
              tc_commit(&k_empty[(j + 1) & 1]);
            }
          }
          if (!mbar_wait(&p_full[0], j & 1, abort, 13)) break;
          tc_fence_after();
          issue_pv(0, j, 1);
          tc_commit(&v_empty[j & 1]);
          if (!kSepP && j + 1 < n_kv) {
            if (!mbar_wait(&k_full[(j + 1) & 1], ((j + 1) >> 1) & 1, abort, 14)) break;
            tc_fence_after();
            issue_s(0, j + 1);
            tc_commit(&k_empty[(j + 1) & 1]);
          }
        }
      }
      for (int j = 0; NG == 2 && ok && j < n_kv; ++j) {
        const bool more = j + 1 < n_kv;
        if (!mbar_wait(&p_half[0], j & 1, abort, 12)) break;
        if (!mbar_wait(&v_full[j & 1], (j >> 1) & 1, abort, 18)) break;
        tc_fence_after();
        issue_pv(0, j, 0);
        if (!mbar_wait(&p_full[0], j & 1, abort, 13)) break;
        tc_fence_after();
        issue_pv(0, j, 1);
        if (more) {
          if (!mbar_wait(&k_full[(j + 1) & 1], ((j + 1) >> 1) & 1, abort, 14)) break;
          tc_fence_after();
          issue_s(0, j + 1);
        }
        if (!mbar_wait(&p_half[1], j & 1, abort, 19)) break;
        tc_fence_after();
        issue_pv(1, j, 0);
        if (!mbar_wait(&p_full[1], j & 1, abort, 15)) break;
        tc_fence_after();
        issue_pv(1, j, 1);
        tc_commit(&v_empty[j & 1]);  // V_j no longer read
        if (more) {
          issue_s(1, j + 1);
          tc_commit(&k_empty[(j + 1) & 1]);  // K_{j+1} no longer read
        }
      }
    }
  } else if (warp >= fwd_soft_warp0<NG>()) {
    // ------------------------------------------------ softmax groups
    const int g = (warp - fwd_soft_warp0<NG>()) >> 2;
    const int qw = warp & 3;
    const int r = qw * 32 + lane;  // row within the query tile == TMEM lane
    const int qrow = q0 + g * TQ + r;
    const uint32_t lane_off = (uint32_t)(qw * 32) << 16;
    const uint32_t t_s = tmem + lane_off + g * 128;
    const uint32_t t_o = tmem + lane_off + kOCol + g * D;
    const uint32_t t_p = kSepP ? tmem + lane_off + kPCol : t_s;  // packed P
    float m_used = -INFINITY, l = 0.f;
    bool ok = n_kv > 0;
    for (int j = 0; ok && j < n_kv; ++j) {
      if (!mbar_wait(&s_full[g], j & 1, abort, 16)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const bool diag = p.causal && (j * TK + TK - 1 > q0 + g * TQ + diag_shift);
      const int kmax = qrow + diag_shift - j * TK;  // columns > kmax are masked
      // pass 1: row max of the scaled scores (log2 domain)
      float mx = -INFINITY;
      {
        uint32_t sv[TK];
        tmem_ld32(t_s + 0, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
        tmem_ld32(t_s + 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
        tmem_ld32(t_s + 64, *reinterpret_cast<uint32_t(*)[32]>(&sv[64]));
        tmem_ld32(t_s + 96, *reinterpret_cast<uint32_t(*)[32]>(&sv[96]));
        tmem_wait_ld();
        // Eight independent chains of 3-input maxima (a single fmaxf chain over 128
        // columns is latency-bound with two softmax warps per scheduler).
        auto row_max = [&](auto val) {
          float m[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) m[k] = fmaxf(val(2 * k), val(2 * k + 1));
#pragma unroll
          for (int i = 16; i < TK; i += 16)
#pragma unroll
            for (int k = 0; k < 8; ++k) m[k] = fmax3(m[k], val(i + 2 * k), val(i + 2 * k + 1));
          return fmaxf(fmax3(m[0], m[1], m[2]), fmax3(fmax3(m[3], m[4], m[5]), m[6], m[7]));
        };
        if (diag || !(p.scale_log2 > 0.f)) {
          mx = row_max([&](int i) {
            return (diag && i > kmax) ? kMaskValue : __uint_as_float(sv[i]) * p.scale_log2;
          });
        } else {
          // scale > 0: max commutes with the scaling
          mx = row_max([&](int i) { return __uint_as_float(sv[i]); }) * p.scale_log2;
        }
      }
      if (kSepP && j > 0) {
        // P V(j - 1) has read P(j - 1) (its columns are rewritten below) and O is final
        // for the rescale
        if (!mbar_wait(&pv_done[g], (j - 1) & 1, abort, 21)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      const float m_new = fmaxf(m_used, mx);
      const bool need = m_new > m_used + kRescaleLog2;
      if (__any_sync(0xffffffffu, need)) {
        const float alpha = need ? ex2_approx(m_used - m_new) : 1.0f;
        if (j > 0) {
          // O_g holds P V up to tile j-1: wait for it, then rescale in TMEM
          if (!mbar_wait(&pv_done[g], (j - 1) & 1, abort, 17)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            uint32_t ov[32];
            tmem_ld32(t_o + c * 32, ov);
            tmem_wait_ld();
            const uint64_t a2 = f2_make(alpha, alpha);
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
              const uint64_t o2 = f2_mul(f2_make_bits(ov[i], ov[i + 1]), a2);
              ov[i] = (uint32_t)o2;
              ov[i + 1] = (uint32_t)(o2 >> 32);
            }
            tmem_st32(t_o + c * 32, ov);
          }
          tmem_wait_st();
        }
        if (need) {
          l *= alpha;
          m_used = m_new;
        }
      }
      // pass 2, two halves of 64 keys: p = 2^(x - m) rounded to the input dtype,
      // packed in pairs into S columns [0, 64) (already consumed).
      // Column pairs go through the packed f32x2 pipe: x = s * scale - m (FFMA2)
      // and two running pair sums (FADD2); exponentials stay scalar.
      const uint64_t sc2 = f2_make(p.scale_log2, p.scale_log2);
      const uint64_t nm2 = f2_make(-m_used, -m_used);
      uint64_t rs2[2] = {f2_make(0.f, 0.f), f2_make(0.f, 0.f)};
      auto pass2 = [&](auto masked) {
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t sv[64];
          tmem_ld32(t_s + half * 64, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
          tmem_ld32(t_s + half * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
          tmem_wait_ld();
          if (kSepP && half == 1) {  // all of S(j) is in registers: S(j + 1) may overwrite it
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_free[g]);
          }
          uint32_t pk[32];
#pragma unroll
          for (int i = 0; i < 64; i += 2) {
            const uint64_t x2 = f2_fma(f2_make_bits(sv[i], sv[i + 1]), sc2, nm2);
            float x0 = f2_lo(x2), x1 = f2_hi(x2);
            if constexpr (decltype(masked)::value) {
              const int col = half * 64 + i;
              x0 = col > kmax ? -INFINITY : x0;
              x1 = col + 1 > kmax ? -INFINITY : x1;
            }
            const float p0 = ex2_approx(x0);
            const float p1 = ex2_approx(x1);
            rs2[(i >> 1) & 1] = f2_add(rs2[(i >> 1) & 1], f2_make(p0, p1));
            pk[i / 2] = BF16 ? pack_bf16x2(p0, p1) : pack_f16x2(p0, p1);
          }
          tmem_st32(t_p + half * 32, pk);
          if (half == 0) {
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_half[g]);
          }
        }
      };
      if (diag)
        pass2(std::true_type{});
      else
        pass2(std::false_type{});
      {
        const uint64_t r2 = f2_add(rs2[0], rs2[1]);
        l += f2_lo(r2) + f2_hi(r2);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[g]);
    }
    // epilogue: O / l -> global, lse
    if (ok && n_kv > 0 && mbar_wait(&pv_done[g], (n_kv - 1) & 1, abort, 18)) {
      tc_fence_after();
      const float inv = 1.0f / l;
      typedef typename std::conditional<BF16, __nv_bfloat16, __half>::type T;
      T* orow = reinterpret_cast<T*>(p.o) + p.lo.row(bh, qrow);
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t ov[32];
        tmem_ld32(t_o + c * 32, ov);
        tmem_wait_ld();
        if (qrow < p.sq) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 v;
            const float* f = reinterpret_cast<const float*>(&ov[i]);
            if constexpr (BF16) {
              v.x = pack_bf16x2(f[0] * inv, f[1] * inv);
              v.y = pack_bf16x2(f[2] * inv, f[3] * inv);
              v.z = pack_bf16x2(f[4] * inv, f[5] * inv);
              v.w = pack_bf16x2(f[6] * inv, f[7] * inv);
            } else {
              v.x = pack_f16x2(f[0] * inv, f[1] * inv);
              v.y = pack_f16x2(f[2] * inv, f[3] * inv);
              v.z = pack_f16x2(f[4] * inv, f[5] * inv);
              v.w = pack_f16x2(f[6] * inv, f[7] * inv);
            }
            *reinterpret_cast<uint4*>(orow + c * 32 + i) = v;
          }
        }
      }
      if (qrow < p.sq) p.lse[(int64_t)bh * p.sq + qrow] = (m_used + log2f(l)) * kLn2;
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, fwd_tmem_cols<NG>());
  }
}

// ===========================================================================
// Tensor-core backward: one kernel template for dK/dV and for dQ
// ===========================================================================
//
// A CTA keeps a 128-row "stationary" pair X1, X2 in shared memory and sweeps
// 64-row "streaming" tiles Y1, Y2 (2-slot TMA ring):
//   dK/dV (IS_DKV): X1 = K, X2 = V (128 keys);  Y1 = Q, Y2 = dO (64 queries),
//                   plus the 64 queries' lse and delta (TMA, zero-filled past sq)
//   dQ            : X1 = Q, X2 = dO (128 queries); Y1 = K, Y2 = V (64 keys)
// Per streaming tile i (warp 1, one lane, kind::f16, f32 accumulators in TMEM):
//   T1 = X1 Y1^T   (dK/dV: S^T;  dQ: S)      128 x 64, TMEM buffer i % 2
//   T2 = X2 Y2^T   (dK/dV: dP^T; dQ: dP)     128 x 64, TMEM buffer i % 2
// Elementwise warpgroup i % 2 (warps 4-7 or 8-11, one thread per X row = TMEM
// lane; the two groups ping-pong over the tiles) forms
//   P = exp(scale*S - lse) (causal mask with the finite MASK_VALUE),
//   dS = P * (dP - delta),
// rounds both to the input dtype (flash_attention.py:210-211, :234) and writes
// them back into the first 32 columns of T1 / T2 as packed pairs; warp 1 then
// accumulates with TS-form MMAs (A read from TMEM)
//   dK/dV: dV += P^T dO, dK += dS^T Q      (B operands = the same Y tiles read
//   dQ   : dQ += dS K                        MN-major: no transposed copies)
// MMAs issued by one thread run in issue order, so T(i+2) (which overwrites
// those columns) is issued after the accumulation of tile i.  With P and dS in
// TMEM the streaming ring has 4 slots, so TMA loads run two tiles ahead.
// After the last tile the two groups scale dK / dQ by `scale`
// (flash_attention.py:220, :243) and store.  No atomics: each CTA owns its
// output rows (grids of flash_attention.py:253-306).

constexpr int BX = 128;  // stationary rows
constexpr int BY = 64;   // streaming rows
constexpr int kBwdThreads = 384;  // 12 warps

constexpr int kYStages = 4;  // streaming TMA ring depth

template <int D>
struct BwdSmem {
  static constexpr int kChunks = D / 64;
  static constexpr int kXBytes = BX * D * 2;  // one stationary tile
  static constexpr int kYBytes = BY * D * 2;  // one streaming tile
  static constexpr int kStatBytes = 2 * BY * 4;  // lse, delta of the streaming rows
  static constexpr int kStageBytes = 2 * kYBytes + 1024;  // Y1, Y2, stats (padded to 1 KiB)
  static constexpr int kX1Off = 0;
  static constexpr int kX2Off = kXBytes;
  static constexpr int kYOff = 2 * kXBytes;
  // dK/dV with a dS output: one 128-key x 64-query bf16 staging tile (32 rows per
  // elementwise warp, 128-byte swizzle) that the TMA store reads; the two
  // elementwise groups hand it to each other tile by tile.
  static constexpr int kStgOff = kYOff + kYStages * kStageBytes;
  // D = 64 leaves room for one staging tile per group (no hand-off wait)
  static constexpr bool kOwnStg = D == 64;
  static constexpr int kStgBytes = BX * BY * 2 * (kOwnStg ? 2 : 1);
  static constexpr int kBarOff = kStgOff + kStgBytes;
  // x_full, y_full[S], y_empty[S], t_full[2], e_full[2], acc_full, x_tmem, stg_free
  static constexpr int kNumBars = 2 * kYStages + 8;
  static constexpr int kTotal = 1024 + kBarOff + kNumBars * 8 + 16;
};

struct BwdParams {
  int sq, sk;
  float scale;
  float scale_log2;
  int causal;
  const float* lse;    // dQ: per-row statistics
  const float* delta;
  void* out0;  // dK/dV: dK; dQ: dQ
  void* out1;  // dK/dV: dV
  Bhsd l0, l1;  // layouts of out0, out1
  int n_x_tiles;
  int bh0;          // first batch*head slice of this launch (grid.y counts from it)
  void* ds;         // dK/dV only, optional: dS^T [slice][key][ds_ld] in the input dtype
  int64_t ds_ld;    // elements per key row (sq rounded up to 64)
  int64_t ds_slice; // elements per slice
};

template <int D, bool BF16, bool IS_DKV>
__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap tx1, const __grid_constant__ CUtensorMap tx2,
                       const __grid_constant__ CUtensorMap ty1, const __grid_constant__ CUtensorMap ty2,
                       const __grid_constant__ CUtensorMap tlse, const __grid_constant__ CUtensorMap tdelta,
                       const __grid_constant__ CUtensorMap tds, const BwdParams p) {
  using L = BwdSmem<D>;
  typedef typename std::conditional<BF16, __nv_bfloat16, __half>::type T;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* x_full = bars + 0;
  uint64_t* y_full = bars + 1;
  uint64_t* y_empty = bars + 1 + kYStages;
  uint64_t* t_full = bars + 1 + 2 * kYStages;
  uint64_t* e_full = t_full + 2;
  uint64_t* acc_full = e_full + 2;
  uint64_t* x_tmem = acc_full + 1;  // dQ: Q and dO copied into TMEM
  uint64_t* stg_free = x_tmem + 1;  // dS staging tile released by the previous tile's warps
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::kNumBars);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Heaviest tiles first: under a causal mask early key tiles (dK/dV) and late
  // query tiles (dQ) see the most streaming tiles.
  const int xt = IS_DKV ? (int)blockIdx.x : p.n_x_tiles - 1 - (int)blockIdx.x;
  const int bh = p.bh0 + (int)blockIdx.y;
  const int hh = bh % p.l0.nh, bb = bh / p.l0.nh;  // TMA coordinates of the slice
  const int x0 = xt * BX;
  const int x_len = IS_DKV ? p.sk : p.sq;  // rows of the stationary operand
  const int y_len = IS_DKV ? p.sq : p.sk;  // rows of the streaming operand
  const int diag_shift = p.sk - p.sq;      // causal: key <= query + diag_shift
  // Streaming tiles [j0, j1) this CTA needs.
  int j0 = 0, j1 = (y_len + BY - 1) / BY;
  if (p.causal) {
    if (IS_DKV) {
      const int q_first = max(0, x0 - diag_shift);  // first query that sees key x0
      j0 = q_first / BY;
    } else {
      const int last_key = min(p.sk - 1, x0 + BX - 1 + diag_shift);
      j1 = last_key < 0 ? 0 : last_key / BY + 1;
    }
  }
  const int n_y = max(0, j1 - j0);

  if (threadIdx.x == 0) {
    mbar_init(x_full, 1);
    mbar_init(acc_full, 1);
    mbar_init(x_tmem, 4);
    mbar_init(stg_free, 4);
    for (int i = 0; i < kYStages; ++i) {
      mbar_init(&y_full[i], 1);
      mbar_init(&y_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&t_full[i], 1);
      mbar_init(&e_full[i], 4);  // one arrival per elementwise warp of the group
    }
    *abort = 0;
    fence_mbar_init();
  }
  // The stationary tiles and the first streaming stages (all slots still free)
  // are requested before the TMEM allocation below, which waits for the SM's
  // previous CTA to release its columns: they stream in under that CTA's tail.
  auto load_y = [&](int i) {
    const int s = i % kYStages;
    uint8_t* y1 = smem + L::kYOff + s * L::kStageBytes;
    uint8_t* y2 = y1 + L::kYBytes;
    mbar_arrive_expect_tx(&y_full[s], 2 * L::kYBytes + (IS_DKV ? L::kStatBytes : 0));
    const int yrow = (j0 + i) * BY;
#pragma unroll
    for (int c = 0; c < L::kChunks; ++c) {
      tma_load_4d(y1 + c * (BY * 128), &ty1, &y_full[s], c * 64, yrow, hh, bb);
      tma_load_4d(y2 + c * (BY * 128), &ty2, &y_full[s], c * 64, yrow, hh, bb);
    }
    if constexpr (IS_DKV) {
      float* st = reinterpret_cast<float*>(y2 + L::kYBytes);
      tma_load_2d(st, &tlse, &y_full[s], yrow, bh);
      tma_load_2d(st + BY, &tdelta, &y_full[s], yrow, bh);
    }
  };
  const int n_pre = min(n_y, kYStages);
  if (threadIdx.x == 0 && n_y > 0) {
    tma_prefetch_desc(&tx1);
    tma_prefetch_desc(&tx2);
    tma_prefetch_desc(&ty1);
    tma_prefetch_desc(&ty2);
    pdl_wait();  // the inputs may come from the previous kernel in the stream
    mbar_arrive_expect_tx(x_full, 2 * L::kXBytes);
#pragma unroll
    for (int c = 0; c < L::kChunks; ++c) {
      tma_load_4d(smem + L::kX1Off + c * (BX * 128), &tx1, x_full, c * 64, x0, hh, bb);
      tma_load_4d(smem + L::kX2Off + c * (BX * 128), &tx2, x_full, c * 64, x0, hh, bb);
    }
    for (int i = 0; i < n_pre; ++i) load_y(i);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_launch_dependents();  // every CTA holds its TMEM before the next kernel is scheduled
  pdl_wait();
  // TMEM columns: T1[2] at 0/64, T2[2] at 128/192, acc0 at 256, then
  //   dK/dV: acc1 at 256 + D;
  //   dQ:    Q and dO as packed 16-bit pairs (A operands of the T MMAs, read from
  //          TMEM so those small-N MMAs only stream the K/V tile from shared
  //          memory) at 256 + D and 256 + D + D/2.
  const uint32_t t_acc0 = tmem + 256;
  const uint32_t t_acc1 = tmem + 256 + D;
  const uint32_t t_xq = tmem + 256 + D;
  const uint32_t t_xdo = tmem + 256 + D + D / 2;

  if (warp == 0) {
    if (lane == 0 && n_y > 0) {
      for (int i = n_pre; i < n_y; ++i) {
        if (!mbar_wait(&y_empty[i % kYStages], ((i / kYStages) & 1) ^ 1, abort, 20)) break;
        load_y(i);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && n_y > 0) {
      constexpr uint32_t idesc_t = make_idesc_f16(BX, BY, BF16, false, false);
      constexpr uint32_t idesc_a = make_idesc_f16(BX, D, BF16, false, true);
      const uint32_t sx1 = smem_u32(smem + L::kX1Off);
      const uint32_t sx2 = smem_u32(smem + L::kX2Off);
      bool ok = mbar_wait(x_full, 0, abort, 21);
      if constexpr (!IS_DKV) ok = ok && mbar_wait(x_tmem, 0, abort, 29);
      // Descriptors are built once; each MMA adds a compile-time byte offset.
      const uint64_t dx1 = make_sdesc(sx1, 16, 1024);
      const uint64_t dx2 = make_sdesc(sx2, 16, 1024);
      const uint64_t dy_k = make_sdesc(smem_u32(smem + L::kYOff), 16, 1024);          // Y, K-major
      const uint64_t dy_mn = make_sdesc(smem_u32(smem + L::kYOff), BY * 128, 1024);   // Y, MN-major
      auto issue_t = [&](int i) -> bool {
        const int s = i % kYStages, b = i & 1;
        if (!mbar_wait(&y_full[s], (i / kYStages) & 1, abort, 22)) return false;
        tc_fence_after();
        const uint64_t dy1 = sdesc_at(dy_k, s * L::kStageBytes);
        const uint64_t dy2 = sdesc_at(dy1, L::kYBytes);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t xo = (kk >> 2) * (BX * 128) + (kk & 3) * 32;
          const uint32_t yo = (kk >> 2) * (BY * 128) + (kk & 3) * 32;
          if constexpr (IS_DKV) {
            tc_mma_f16_ss(tmem + b * 64, sdesc_at(dx1, xo), sdesc_at(dy1, yo), idesc_t, kk != 0);
            tc_mma_f16_ss(tmem + 128 + b * 64, sdesc_at(dx2, xo), sdesc_at(dy2, yo), idesc_t, kk != 0);
          } else {
            tc_mma_f16_ts(tmem + b * 64, t_xq + kk * 8, sdesc_at(dy1, yo), idesc_t, kk != 0);
            tc_mma_f16_ts(tmem + 128 + b * 64, t_xdo + kk * 8, sdesc_at(dy2, yo), idesc_t, kk != 0);
          }
        }
        tc_commit(&t_full[b]);
        return true;
      };
      auto issue_acc = [&](int i) -> bool {
        const int s = i % kYStages, b = i & 1;
        if (!mbar_wait(&e_full[b], (i >> 1) & 1, abort, 24)) return false;
        tc_fence_after();
        const uint64_t dm1 = sdesc_at(dy_mn, s * L::kStageBytes);
        const uint64_t dm2 = sdesc_at(dm1, L::kYBytes);
        const uint32_t tP = tmem + b * 64;         // P (dK/dV only): T1 columns [0, 32)
        const uint32_t tdS = tmem + 128 + b * 64;  // dS: T2 columns [0, 32)
#pragma unroll
        for (int kk = 0; kk < BY / 16; ++kk) {
          const uint32_t yo = kk * 2048;  // MN-major Y: 16 rows per step
          const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
          if constexpr (IS_DKV) {
            // dV += P^T dO   (acc1),   dK += dS^T Q  (acc0)
            tc_mma_f16_ts(t_acc1, tP + kk * 8, sdesc_at(dm2, yo), idesc_a, acc);
            tc_mma_f16_ts(t_acc0, tdS + kk * 8, sdesc_at(dm1, yo), idesc_a, acc);
          } else {
            // dQ += dS K  (acc0)
            tc_mma_f16_ts(t_acc0, tdS + kk * 8, sdesc_at(dm1, yo), idesc_a, acc);
          }
        }
        tc_commit(&y_empty[s]);
        return true;
      };
      if (ok) ok = issue_t(0);
      if (ok && n_y > 1) ok = issue_t(1);
      for (int i = 0; ok && i < n_y; ++i) {
        ok = issue_acc(i);
        if (ok && i + 2 < n_y) ok = issue_t(i + 2);
      }
      tc_commit(acc_full);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------ elementwise warpgroups
    const int g = (warp - 4) >> 2;  // group g handles tiles i with i % 2 == g
    const int qw = warp & 3;
    const int r = qw * 32 + lane;  // stationary row == TMEM lane
    const int xrow = x0 + r;
    const uint32_t lane_off = (uint32_t)(qw * 32) << 16;
    const uint32_t t_t1 = tmem + lane_off + g * 64;
    const uint32_t t_t2 = tmem + lane_off + 128 + g * 64;
    if constexpr (!IS_DKV) {
      // Group 0 moves this CTA's Q and dO rows from the swizzled shared tiles into
      // TMEM (one row per lane, 16-bit pairs along d) once, before any T MMA.
      if (g == 0 && n_y > 0) {
        if (mbar_wait(x_full, 0, abort, 30)) {
#pragma unroll
          for (int m = 0; m < 2; ++m) {
            const uint8_t* xs = smem + (m == 0 ? L::kX1Off : L::kX2Off);
            uint32_t w[D / 2];
#pragma unroll
            for (int ch = 0; ch < D / 64; ++ch)
#pragma unroll
              for (int gr = 0; gr < 8; ++gr) {
                const uint4 v = *reinterpret_cast<const uint4*>(xs + ch * (BX * 128) + swz128(r, gr));
                w[ch * 32 + gr * 4 + 0] = v.x;
                w[ch * 32 + gr * 4 + 1] = v.y;
                w[ch * 32 + gr * 4 + 2] = v.z;
                w[ch * 32 + gr * 4 + 3] = v.w;
              }
            const uint32_t dst = (m == 0 ? t_xq : t_xdo) + lane_off;
#pragma unroll
            for (int c32 = 0; c32 < D / 64; ++c32)
              tmem_st32(dst + c32 * 32, *reinterpret_cast<uint32_t(*)[32]>(&w[c32 * 32]));
          }
          tmem_wait_st();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(x_tmem);
      }
    }
    // dQ: this row's statistics (rows past sq are masked below)
    float row_lse2 = 0.f, row_delta = 0.f;
    if (!IS_DKV && xrow < p.sq) {
      row_lse2 = p.lse[(int64_t)bh * p.sq + xrow] * kLog2e;
      row_delta = p.delta[(int64_t)bh * p.sq + xrow];
    }
    bool ok = n_y > 0;
    for (int i = g; ok && i < n_y; i += 2) {
      const int ph = (i >> 1) & 1;
      const int y0 = (j0 + i) * BY;
      if (!mbar_wait(&t_full[g], ph, abort, 25)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t a[BY], b[BY];
      tmem_ld32(t_t1, *reinterpret_cast<uint32_t(*)[32]>(&a[0]));
      tmem_ld32(t_t1 + 32, *reinterpret_cast<uint32_t(*)[32]>(&a[32]));
      tmem_ld32(t_t2, *reinterpret_cast<uint32_t(*)[32]>(&b[0]));
      tmem_ld32(t_t2 + 32, *reinterpret_cast<uint32_t(*)[32]>(&b[32]));
      const float* st = nullptr;
      if constexpr (IS_DKV) {
        // the stage's lse / delta (already landed: T(i) was computed from this stage)
        const int s = i % kYStages;
        if (!mbar_wait(&y_full[s], (i / kYStages) & 1, abort, 26)) {
          ok = false;
          break;
        }
        st = reinterpret_cast<const float*>(smem + L::kYOff + s * L::kStageBytes + 2 * L::kYBytes);
      }
      tmem_wait_ld();
      // Masking is tile-uniform except on the causal diagonal and past sq; the
      // exponent input is set to -inf where masked (ex2.approx.ftz(-inf) = +0),
      // so the loop has no per-element branches.
      bool need_mask;
      if constexpr (IS_DKV)
        need_mask = (y0 + BY > p.sq) || (p.causal && x0 + BX - 1 > y0 + diag_shift);
      else
        need_mask = (x0 + BX > p.sq) || (p.causal && y0 + BY - 1 > x0 + diag_shift);
      uint32_t pp[BY / 2], dd[BY / 2];
      auto body = [&](auto masked) {
#pragma unroll
        for (int e = 0; e < BY; e += 2) {
          float pv[2], dv[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int c = e + u;  // streaming column
            float l2, dl;
            if constexpr (IS_DKV) {
              l2 = st[c] * kLog2e;
              dl = st[BY + c];
            } else {
              l2 = row_lse2;
              dl = row_delta;
            }
            float x = fmaf(__uint_as_float(a[c]), p.scale_log2, -l2);
            if constexpr (decltype(masked)::value) {
              const int key = IS_DKV ? xrow : y0 + c;
              const int qry = IS_DKV ? y0 + c : xrow;
              const bool valid = qry < p.sq && !(p.causal && key > qry + diag_shift);
              x = valid ? x : -INFINITY;
            }
            const float pr = ex2_approx(x);
            pv[u] = pr;
            dv[u] = pr * (__uint_as_float(b[c]) - dl);
          }
          pp[e / 2] = BF16 ? pack_bf16x2(pv[0], pv[1]) : pack_f16x2(pv[0], pv[1]);
          dd[e / 2] = BF16 ? pack_bf16x2(dv[0], dv[1]) : pack_f16x2(dv[0], dv[1]);
        }
      };
      if (need_mask)
        body(std::true_type{});
      else
        body(std::false_type{});
      if constexpr (IS_DKV) tmem_st32(t_t1, pp);
      tmem_st32(t_t2, dd);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&e_full[g]);
      if constexpr (IS_DKV) {
        // dS^T rows (these 32 keys x the tile's 64 queries) for the dQ-from-dS
        // kernel, off the MMA's critical path: the accumulation MMAs of this
        // tile are already released.  Staged in shared memory (swizzled rows,
        // conflict-free) and written by one TMA store per warp.
        if (p.ds != nullptr) {
          if constexpr (L::kOwnStg) {
            if (lane == 0) bulk_wait_group_read0();  // this warp's store of two tiles ago
            __syncwarp();
          } else if (i > 0 && !mbar_wait(stg_free, (i - 1) & 1, abort, 31)) {
            ok = false;
            break;
          }
          uint8_t* stg = smem + L::kStgOff + (L::kOwnStg ? g * (BX * BY * 2) : 0) + qw * 4096;
          uint8_t* row = stg + lane * 128;
#pragma unroll
          for (int v = 0; v < BY / 8; ++v)
            *reinterpret_cast<uint4*>(row + ((v ^ (lane & 7)) << 4)) =
                make_uint4(dd[4 * v], dd[4 * v + 1], dd[4 * v + 2], dd[4 * v + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            // dS^T is stored in 64-key x 64-query blocks (8 KiB contiguous):
            // coordinates (query in block, key in block, query block, key block)
            const int key = x0 + qw * 32;
            tma_store_4d(&tds, stg, 0, key & 63, y0 >> 6, (int)blockIdx.y * (p.sk >> 6) + (key >> 6));
            bulk_commit_group();
            if constexpr (!L::kOwnStg) {
              bulk_wait_group_read0();  // staging read: hand it to the other group
              mbar_arrive(stg_free);
            }
          }
          __syncwarp();
        }
      }
    }
    if constexpr (IS_DKV) {
      if (p.ds != nullptr && lane == 0) bulk_wait_group0();  // dS writes complete before exit
    }
    // epilogue: dK/dV -> group 0 stores dK, group 1 stores dV; dQ -> column halves
    if (ok && n_y > 0 && mbar_wait(acc_full, 0, abort, 28)) {
      tc_fence_after();
      const bool row_ok = xrow < x_len;
      const int64_t orow = ((IS_DKV && g == 1) ? p.l1 : p.l0).row(bh, xrow);
      T* out = reinterpret_cast<T*>((IS_DKV && g == 1) ? p.out1 : p.out0) + orow;
      const uint32_t src = (IS_DKV && g == 1) ? t_acc1 : t_acc0;
      const float mul = (IS_DKV && g == 1) ? 1.0f : p.scale;
      const int c_begin = IS_DKV ? 0 : g * (D / 2);
      const int c_end = IS_DKV ? D : (g + 1) * (D / 2);
      for (int c0 = c_begin; c0 < c_end; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(src + lane_off + c0, v);
        tmem_wait_ld();
        if (row_ok) {
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            uint4 w;
            const float* f = reinterpret_cast<const float*>(&v[e]);
            w.x = BF16 ? pack_bf16x2(f[0] * mul, f[1] * mul) : pack_f16x2(f[0] * mul, f[1] * mul);
            w.y = BF16 ? pack_bf16x2(f[2] * mul, f[3] * mul) : pack_f16x2(f[2] * mul, f[3] * mul);
            w.z = BF16 ? pack_bf16x2(f[4] * mul, f[5] * mul) : pack_f16x2(f[4] * mul, f[5] * mul);
            w.w = BF16 ? pack_bf16x2(f[6] * mul, f[7] * mul) : pack_f16x2(f[6] * mul, f[7] * mul);
            *reinterpret_cast<uint4*>(out + c0 + e) = w;
          }
        }
      }
    } else if (ok && n_y == 0 && xrow < x_len) {
      // no streaming tile reaches these rows (not reachable for causal sq == sk): zeros
      const int64_t orow = ((IS_DKV && g == 1) ? p.l1 : p.l0).row(bh, xrow);
      T* out = reinterpret_cast<T*>((IS_DKV && g == 1) ? p.out1 : p.out0) + orow;
      const int c_begin = IS_DKV ? 0 : g * (D / 2);
      const int c_end = IS_DKV ? D : (g + 1) * (D / 2);
      for (int c = c_begin; c < c_end; ++c) out[c] = DT<T>::from_f(0.f);
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ===========================================================================
// dK/dV with 128-query streaming tiles (tensor cores, every product N >= 128)
// ===========================================================================
//
// Same work as the dK/dV instance above (flash_attention.py:197-221, one CTA per
// 128-key tile, no atomics) with 128-query streaming tiles, so that S^T = K Q^T
// and dP^T = V dO^T are 128 x 128 products: a 128 x 64 tcgen05.mma takes as long
// as a 128 x 128 one, so the 64-query tiles spent half the tensor time of their
// two T products.  The 512 TMEM columns hold one S^T, one dP^T and the dK, dV
// accumulators -- no room to double-buffer T -- so the two 128-column regions
// R0, R1 swap roles every tile (S^T(i) in R(i % 2), dP^T(i) in the other) and
// the elementwise work is split in two phases:
//   EW-a(i): P = exp(scale S - lse) from S^T (registers, f32) -> P^T packed into
//            its own S^T columns (TS operand of dV += P^T dO)
//   EW-b(i): reads dP^T(i) (releasing its region), dS = P (dP - delta) -> bf16
//            dS^T packed into the other half of its S^T columns (TS operand of
//            dK += dS^T Q), then into a 128-byte-swizzled shared tile that the TMA
//            store of dS^T (for the dQ-from-dS kernel) reads -- after the dK
//            operand is published, so the store is off the MMA's path.
// MMA order per tile:  dV(i) part 0 | S(i+1) | dV(i) part 1 | dK(i) | dP(i+1).
// S(i+1) goes into dP(i)'s region as soon as EW-b(i) holds dP(i) in registers, so
// EW-a(i+1) starts right after EW-b(i); dP(i+1) overwrites S(i)'s region after dV(i)
// and dK(i) (issued before it; tcgen05.mma executes in issue order) have read P(i)
// and dS(i) there.
// Warps: 0 TMA producer, 1 TMEM owner + MMA lane, 2-9 elementwise: warp w
// handles TMEM lanes 32 (w % 4) .. +31 (key rows) and query columns
// [64 h, 64 h + 64) of each tile, h = (w - 2) / 4.
// TMEM: R0 [0,128), R1 [128,256) (P^T packed at +[0,32) and +[64,96) of the S^T
// region, dS^T at +[32,64) and +[96,128)), dV [256, 256+D), dK [256+D, 256+2D).

constexpr int kWideY = 128;                 // streaming rows (queries) per tile
constexpr int kWideThreads = 320;           // 10 warps

template <int D>
struct WideSmem {
  static constexpr int kChunks = D / 64;
  static constexpr int kXBytes = BX * D * 2;            // K or V tile
  static constexpr int kYBytes = kWideY * D * 2;        // Q or dO tile
  static constexpr int kStages = D == 64 ? 3 : 2;
  static constexpr int kStageBytes = 2 * kYBytes + 1024;  // Q, dO, lse + delta (128 f32 each)
  static constexpr int kX1Off = 0;
  static constexpr int kX2Off = kXBytes;
  static constexpr int kYOff = 2 * kXBytes;
  static constexpr int kStgOff = kYOff + kStages * kStageBytes;  // dS^T: 2 x [128 keys x 64 queries]
  static constexpr int kDataBytes = kStgOff + BX * kWideY * 2;
  // x_full, y_full[S], y_empty[S], s_full, dp_full, p_full, dp_free, ds_full, acc_full, p_half
  static constexpr int kNumBars = 2 * kStages + 8;
  static constexpr int kBarBytes = kNumBars * 8 + 8;  // + TMEM slot + abort flag
  static_assert(kBarBytes <= 128, "barrier block must fit the alignment slack rule");
  // Data is placed at the first 1024-byte boundary; the barrier block goes into the
  // slack before it when that is >= 128 bytes, else right after the data (the
  // slack is then < 128, and 1024 extra bytes cover both cases).
  static constexpr int kTotal = kDataBytes + 1024;
};

// Bounded wait that ignores the abort flag: used to drain this CTA's own MMAs
// before TMEM is released on any path.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (!mbar_try_wait(bar, parity)) {
    if ((++spins & 255u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) {
      report_timeout(40);
      return;
    }
  }
}

template <int D, bool BF16>
__global__ void __launch_bounds__(kWideThreads, 1)
    attn_dkv_wide_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                         const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tdo,
                         const __grid_constant__ CUtensorMap tlse, const __grid_constant__ CUtensorMap tdelta,
                         const __grid_constant__ CUtensorMap tds, const BwdParams p) {
  using L = WideSmem<D>;
  constexpr int S = L::kStages;
  typedef typename std::conditional<BF16, __nv_bfloat16, __half>::type T;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem - smem_raw >= 128 ? smem_raw : smem + L::kDataBytes);
  uint64_t* x_full = bars + 0;
  uint64_t* y_full = bars + 1;
  uint64_t* y_empty = bars + 1 + S;
  uint64_t* s_full = bars + 1 + 2 * S;
  uint64_t* dp_full = s_full + 1;
  uint64_t* p_full = s_full + 2;
  uint64_t* dp_free = s_full + 3;
  uint64_t* ds_full = s_full + 4;
  uint64_t* acc_full = s_full + 5;
  uint64_t* p_half = s_full + 6;  // P^T of each warp's first 32 query columns written
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::kNumBars);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int ktile, slice;
  batched_order(p.n_x_tiles, (int)gridDim.y, ktile, slice);  // key block 0 (most causal tiles) first
  const int bh = p.bh0 + slice;
  const int hh = bh % p.l0.nh, bb = bh / p.l0.nh;
  const int x0 = ktile * BX;
  const int diag_shift = p.sk - p.sq;
  int j0 = 0;
  const int j1 = (p.sq + kWideY - 1) / kWideY;
  if (p.causal) j0 = max(0, x0 - diag_shift) / kWideY;
  const int n_y = max(0, j1 - j0);

  if (threadIdx.x == 0) {
    mbar_init(x_full, 1);
    for (int i = 0; i < S; ++i) {
      mbar_init(&y_full[i], 1);
      mbar_init(&y_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(dp_full, 1);
    mbar_init(p_full, 8);   // one arrival per elementwise warp
    mbar_init(p_half, 8);
    mbar_init(dp_free, 8);
    mbar_init(ds_full, 8);
    mbar_init(acc_full, 1);
    *abort = 0;
    fence_mbar_init();
  }
  auto load_y = [&](int i) {
    const int s = i % S;
    uint8_t* y1 = smem + L::kYOff + s * L::kStageBytes;
    uint8_t* y2 = y1 + L::kYBytes;
    mbar_arrive_expect_tx(&y_full[s], 2 * L::kYBytes + 2 * kWideY * 4);
    const int yrow = (j0 + i) * kWideY;
#pragma unroll
    for (int c = 0; c < L::kChunks; ++c) {
      tma_load_4d(y1 + c * (kWideY * 128), &tq, &y_full[s], c * 64, yrow, hh, bb);
      tma_load_4d(y2 + c * (kWideY * 128), &tdo, &y_full[s], c * 64, yrow, hh, bb);
    }
    float* st = reinterpret_cast<float*>(y2 + L::kYBytes);
    tma_load_2d(st, &tlse, &y_full[s], yrow, bh);
    tma_load_2d(st + kWideY, &tdelta, &y_full[s], yrow, bh);
  };
  const int n_pre = min(n_y, S);
  if (threadIdx.x == 0 && n_y > 0) {
    tma_prefetch_desc(&tk);
    tma_prefetch_desc(&tv);
    tma_prefetch_desc(&tq);
    tma_prefetch_desc(&tdo);
    pdl_wait();
    mbar_arrive_expect_tx(x_full, 2 * L::kXBytes);
#pragma unroll
    for (int c = 0; c < L::kChunks; ++c) {
      tma_load_4d(smem + L::kX1Off + c * (BX * 128), &tk, x_full, c * 64, x0, hh, bb);
      tma_load_4d(smem + L::kX2Off + c * (BX * 128), &tv, x_full, c * 64, x0, hh, bb);
    }
    for (int i = 0; i < n_pre; ++i) load_y(i);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_launch_dependents();
  pdl_wait();
  const uint32_t t_dv = tmem + 256;
  const uint32_t t_dk = tmem + 256 + D;

  if (warp == 0) {
    if (lane == 0 && n_y > 0) {
      for (int i = n_pre; i < n_y; ++i) {
        if (!mbar_wait(&y_empty[i % S], ((i / S) & 1) ^ 1, abort, 41)) break;
        load_y(i);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && n_y > 0) {
      constexpr uint32_t idesc_t = make_idesc_f16(BX, kWideY, BF16, false, false);
      constexpr uint32_t idesc_a = make_idesc_f16(BX, D, BF16, false, true);
      const uint64_t dx1 = make_sdesc(smem_u32(smem + L::kX1Off), 16, 1024);
      const uint64_t dx2 = make_sdesc(smem_u32(smem + L::kX2Off), 16, 1024);
      const uint64_t dy_k = make_sdesc(smem_u32(smem + L::kYOff), 16, 1024);
      const uint64_t dy_mn = make_sdesc(smem_u32(smem + L::kYOff), kWideY * 128, 1024);
      bool ok = mbar_wait(x_full, 0, abort, 42);
      // TMEM regions R0 = [0,128), R1 = [128,256) alternate roles: S^T(i) goes to
      // R(i % 2), dP^T(i) to the other.  P^T(i) stays packed in S^T(i)'s region.
      auto region = [&](int i, bool is_s) -> uint32_t { return (((i & 1) ^ (is_s ? 0 : 1)) ? 128u : 0u); };
      auto issue_prod = [&](int i, bool is_s) {
        const uint64_t dy = sdesc_at(dy_k, (i % S) * L::kStageBytes + (is_s ? 0 : L::kYBytes));
        const uint64_t dx = is_s ? dx1 : dx2;
        const uint32_t dst = tmem + region(i, is_s);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t xo = (kk >> 2) * (BX * 128) + (kk & 3) * 32;
          const uint32_t yo = (kk >> 2) * (kWideY * 128) + (kk & 3) * 32;
          tc_mma_f16_ss(dst, sdesc_at(dx, xo), sdesc_at(dy, yo), idesc_t, kk != 0);
        }
        tc_commit(is_s ? s_full : dp_full);
      };
      // dV += P^T(i) dO_i: A = P^T from TMEM, B = dO_i MN-major
      // part 0: query steps kk = 0, 1, 4, 5 (the warps' first 32 columns, p_half);
      // part 1: kk = 2, 3, 6, 7 (p_full)
      auto issue_dv = [&](int i, int part) {
        const uint64_t dm2 = sdesc_at(dy_mn, (i % S) * L::kStageBytes + L::kYBytes);
        const uint32_t pa = tmem + region(i, true);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int kk = (q >> 1) * 4 + part * 2 + (q & 1);
          tc_mma_f16_ts(t_dv, pa + (kk >> 2) * 64 + (kk & 3) * 8, sdesc_at(dm2, kk * 2048), idesc_a,
                        (i > 0 || kk > 0) ? 1u : 0u);
        }
      };
      // dK += dS^T(i) Q_i: A = dS^T packed in S^T(i)'s region (TMEM), B = Q_i MN-major
      auto issue_dk = [&](int i) {
        const uint64_t dm1 = sdesc_at(dy_mn, (i % S) * L::kStageBytes);
        const uint32_t da = tmem + region(i, true) + 32;
#pragma unroll
        for (int kk = 0; kk < kWideY / 16; ++kk)
          tc_mma_f16_ts(t_dk, da + (kk >> 2) * 64 + (kk & 3) * 8, sdesc_at(dm1, kk * 2048), idesc_a,
                        (i > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&y_empty[i % S]);  // Q_i, dO_i, stats no longer read
      };
      // Order per tile i: dV(i) part 0 once the first halves of P(i) are out; S(i+1)
      // as soon as EW-b(i) holds dP(i) (its region); dV(i) part 1; dK(i); dP(i+1) into
      // S(i)'s region after dV(i) and dK(i) (in issue order) have read P(i) and dS(i).
      if (ok && (ok = mbar_wait(&y_full[0], 0, abort, 43))) {
        tc_fence_after();
        issue_prod(0, true);
        issue_prod(0, false);
      }
      for (int i = 0; ok && i < n_y; ++i) {
        const bool more = i + 1 < n_y;
        if (!(ok = mbar_wait(p_half, i & 1, abort, 52))) break;
        tc_fence_after();
        issue_dv(i, 0);
        if (!(ok = mbar_wait(p_full, i & 1, abort, 45))) break;
        if (more) {
          if (!(ok = mbar_wait(dp_free, i & 1, abort, 44))) break;
          if (!(ok = mbar_wait(&y_full[(i + 1) % S], ((i + 1) / S) & 1, abort, 43))) break;
        }
        tc_fence_after();
        if (more) issue_prod(i + 1, true);
        issue_dv(i, 1);
        if (!(ok = mbar_wait(ds_full, i & 1, abort, 46))) break;
        tc_fence_after();
        issue_dk(i);
        if (more) issue_prod(i + 1, false);
      }
      tc_commit(acc_full);
      mbar_drain(acc_full, 0);  // every MMA of this CTA has completed
    }
  } else {
    // ------------------------------------------------ elementwise warps
    const int qw = warp & 3;
    const int h = (warp - 2) >> 2;  // query columns [64 h, 64 h + 64)
    const int r = qw * 32 + lane;   // key row == TMEM lane
    const int xrow = x0 + r;
    const uint32_t lane_off = (uint32_t)(qw * 32) << 16;
    const uint32_t t_col = tmem + lane_off + h * 64;  // + region: S^T (P^T packed in its first 32) / dP^T
    uint8_t* stg = smem + L::kStgOff + h * (BX * 128) + qw * 4096;
    bool ok = true;
    for (int i = 0; ok && i < n_y; ++i) {
      const int ph = i & 1;
      const int y0 = (j0 + i) * kWideY;
      const int s = i % S;
      const uint32_t t_s = t_col + ((i & 1) ? 128u : 0u);
      const uint32_t t_dp = t_col + ((i & 1) ? 0u : 128u);
      const bool need_mask = (y0 + kWideY > p.sq) || (p.causal && x0 + BX - 1 > y0 + diag_shift);
      // ---- EW-a: P = 2^(scale*log2e*S - lse*log2e)
      if (!mbar_wait(s_full, ph, abort, 47) || !mbar_wait(&y_full[s], (i / S) & 1, abort, 48)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float* st = reinterpret_cast<const float*>(smem + L::kYOff + s * L::kStageBytes + 2 * L::kYBytes) + h * 64;
      uint32_t pf[64];
      tmem_ld32(t_s, *reinterpret_cast<uint32_t(*)[32]>(&pf[0]));
      tmem_ld32(t_s + 32, *reinterpret_cast<uint32_t(*)[32]>(&pf[32]));
      tmem_wait_ld();
      {
        // four columns per step: one 16-byte load of lse, packed f32x2 math
        // (each lane rounds exactly like fmaf(s, scale*log2e, -(lse*log2e)))
        const uint64_t sc2 = f2_make(p.scale_log2, p.scale_log2);
        const uint64_t nlog2e2 = f2_make(-kLog2e, -kLog2e);
        auto body_a = [&](auto masked, auto c0) {
#pragma unroll
          for (int c = decltype(c0)::value; c < decltype(c0)::value + 32; c += 4) {
            const float4 l4 = *reinterpret_cast<const float4*>(st + c);
            const uint64_t x01 = f2_fma(f2_make_bits(pf[c], pf[c + 1]), sc2, f2_mul(f2_make(l4.x, l4.y), nlog2e2));
            const uint64_t x23 = f2_fma(f2_make_bits(pf[c + 2], pf[c + 3]), sc2, f2_mul(f2_make(l4.z, l4.w), nlog2e2));
            float x[4] = {f2_lo(x01), f2_hi(x01), f2_lo(x23), f2_hi(x23)};
            if constexpr (decltype(masked)::value) {
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const int qry = y0 + h * 64 + c + u;
                const bool valid = qry < p.sq && !(p.causal && xrow > qry + diag_shift);
                x[u] = valid ? x[u] : -INFINITY;
              }
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) pf[c + u] = __float_as_uint(ex2_approx(x[u]));
          }
        };
        // Two 32-column halves, each published on its own barrier: dV(i) takes the
        // query steps of the first halves (p_half) while the second halves run.
        auto half_a = [&](auto c0, uint64_t* bar) {
          if (need_mask)
            body_a(std::true_type{}, c0);
          else
            body_a(std::false_type{}, c0);
          uint32_t pp[16];
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            const float a0 = __uint_as_float(pf[decltype(c0)::value + c]);
            const float a1 = __uint_as_float(pf[decltype(c0)::value + c + 1]);
            pp[c / 2] = BF16 ? pack_bf16x2(a0, a1) : pack_f16x2(a0, a1);
          }
          tmem_st16(t_s + decltype(c0)::value / 2, pp);
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar);
        };
        half_a(std::integral_constant<int, 0>{}, p_half);
        half_a(std::integral_constant<int, 32>{}, p_full);
      }
      // ---- EW-b: dS = P (dP - delta)
      if (!mbar_wait(dp_full, ph, abort, 49)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // dP^T(i) into registers first: its release (dp_free) lets S(i+1) into the region.
      uint32_t b[64];
      tmem_ld32(t_dp, *reinterpret_cast<uint32_t(*)[32]>(&b[0]));
      tmem_ld32(t_dp + 32, *reinterpret_cast<uint32_t(*)[32]>(&b[32]));
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dp_free);
      // dS(i) goes (a) packed into the free half of S^T(i)'s columns, [64 h + 32,
      // 64 h + 64), where dK(i) reads it as a TMEM operand, and (b) into the shared
      // staging tile for the TMA store of dS^T -- after ds_full, off the MMA's path.
      const bool store_ds = p.ds != nullptr;
      if (store_ds) {
        if (lane == 0) bulk_wait_group_read0();  // this warp's previous store has read the tile
        __syncwarp();
      }
      uint8_t* row = stg + lane * 128;
#pragma unroll
      for (int hb = 0; hb < 2; ++hb) {
        uint32_t dd[16];
#pragma unroll
        for (int e = 0; e < 32; e += 4) {
          const int c = hb * 32 + e;
          const float4 d4 = *reinterpret_cast<const float4*>(st + kWideY + c);
          const uint64_t d01 = f2_mul(f2_make_bits(pf[c], pf[c + 1]),
                                      f2_sub(f2_make_bits(b[c], b[c + 1]), f2_make(d4.x, d4.y)));
          const uint64_t d23 = f2_mul(f2_make_bits(pf[c + 2], pf[c + 3]),
                                      f2_sub(f2_make_bits(b[c + 2], b[c + 3]), f2_make(d4.z, d4.w)));
          dd[e / 2] = BF16 ? pack_bf16x2(f2_lo(d01), f2_hi(d01)) : pack_f16x2(f2_lo(d01), f2_hi(d01));
          dd[e / 2 + 1] = BF16 ? pack_bf16x2(f2_lo(d23), f2_hi(d23)) : pack_f16x2(f2_lo(d23), f2_hi(d23));
        }
        tmem_st16(t_s + 32 + hb * 16, dd);
        if (store_ds) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            const int g16 = hb * 4 + v;  // 16-byte granule of the 128-byte row
            *reinterpret_cast<uint4*>(row + ((g16 ^ (lane & 7)) << 4)) =
                make_uint4(dd[4 * v], dd[4 * v + 1], dd[4 * v + 2], dd[4 * v + 3]);
          }
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(ds_full);
      if (store_ds) {
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          // dS^T in 64-key x 64-query blocks: (query in block, key in block, query block, key block)
          const int key = x0 + qw * 32;
          tma_store_4d(&tds, stg, 0, key & 63, (y0 >> 6) + h, slice * (p.sk >> 6) + (key >> 6));
          bulk_commit_group();
        }
        __syncwarp();
      }
    }
    if (lane == 0) bulk_wait_group0();
    // epilogue: warps with h = 0 store dK (x scale), h = 1 store dV
    if (n_y > 0 && ok && mbar_wait(acc_full, 0, abort, 51)) {
      tc_fence_after();
      const bool row_ok = xrow < p.sk;
      T* out = reinterpret_cast<T*>(h == 0 ? p.out0 : p.out1) + (h == 0 ? p.l0 : p.l1).row(bh, xrow);
      const uint32_t src = (h == 0 ? t_dk : t_dv) + lane_off;
      const float mul = h == 0 ? p.scale : 1.0f;
#pragma unroll
      for (int c0 = 0; c0 < D; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(src + c0, v);
        tmem_wait_ld();
        if (row_ok) {
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            uint4 w;
            const float* f = reinterpret_cast<const float*>(&v[e]);
            w.x = BF16 ? pack_bf16x2(f[0] * mul, f[1] * mul) : pack_f16x2(f[0] * mul, f[1] * mul);
            w.y = BF16 ? pack_bf16x2(f[2] * mul, f[3] * mul) : pack_f16x2(f[2] * mul, f[3] * mul);
            w.z = BF16 ? pack_bf16x2(f[4] * mul, f[5] * mul) : pack_f16x2(f[4] * mul, f[5] * mul);
            w.w = BF16 ? pack_bf16x2(f[6] * mul, f[7] * mul) : pack_f16x2(f[6] * mul, f[7] * mul);
            *reinterpret_cast<uint4*>(out + c0 + e) = w;
          }
        }
      }
    } else if (n_y == 0 && xrow < p.sk) {
      // no query reaches these keys (not reachable when sk % 128 == 0): zeros
      T* out = reinterpret_cast<T*>(h == 0 ? p.out0 : p.out1) + (h == 0 ? p.l0 : p.l1).row(bh, xrow);
      for (int c = 0; c < D; ++c) out[c] = DT<T>::from_f(0.f);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ===========================================================================
// dQ from a materialised dS (tensor cores)
// ===========================================================================
//
// dQ[q, :] = scale * sum_{k <= q} dS[q, k] K[k, :]: with the dK/dV kernel
// writing its bf16 dS^T tiles ([key][query] per slice, the exact values the
// reference rounds before its dQ product, flash_attention.py:234), dQ is a
// batched GEMM  dQ_slice = (dS^T)^T K  -- one tensor-core product per tile
// instead of recomputing S, P, dP and dS (three), and no atomics.  Per work unit
// (128-query tile, slice) the K range stops at the causal diagonal.
//   warp 0      TMA: dS^T boxes {64 queries, 64 keys} (MN-major A) and K boxes
//               {64 d, 64 keys} (MN-major B) into a DQ_STAGES-slot ring;
//   warp 1      TMEM (two D-column accumulators) + one MMA lane, M=128 N=D K=16;
//   warps 2-5   epilogue: tcgen05.ld, x scale, round, 16-byte stores through the
//               dQ layout.
// Persistent: grid = min(units, SMs); slice by slice, heaviest query tile first.
// The host launches it only where every query row sees at least one key (causal
// implies sq == sk on this path), so every unit has K blocks.

constexpr int kDqThreads = 192;

template <int D>
struct DqSmem {
  static constexpr int kABytes = 128 * 64 * 2;  // dS^T: 2 boxes of 64 queries x 64 keys
  static constexpr int kBBytes = 64 * D * 2;    // K: D/64 boxes of 64 d x 64 keys
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = D == 64 ? 8 : 6;
  static constexpr int kBarOff = kStages * kStageBytes;
  static constexpr int kNumBars = 2 * kStages + 4;
  static constexpr int kTotal = 1024 + kBarOff + kNumBars * 8 + 16;
};

struct DqParams {
  int sq, sk, causal, nh;
  float scale;
  int n_q_tiles, n_slices, bh0;
  void* dq;
  Bhsd ldq;
};

template <int D, bool BF16>
__global__ void __launch_bounds__(kDqThreads, 1)
    attn_dq_ds_kernel(const __grid_constant__ CUtensorMap tds, const __grid_constant__ CUtensorMap tk,
                      const DqParams p) {
  using L = DqSmem<D>;
  constexpr int STAGES = L::kStages;
  typedef typename std::conditional<BF16, __nv_bfloat16, __half>::type T;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int units = p.n_q_tiles * p.n_slices;
  const int diag_shift = p.sk - p.sq;
  const int nkb_all = p.sk / 64;  // key blocks per slice in the dS layout
  // unit u: slice u / n_q_tiles, query tile n_q_tiles - 1 - u % n_q_tiles (heaviest
  // first within a slice).  CTAs running at the same time work on the same few
  // slices, so each slice's K tiles are read from HBM once and then hit in L2.
  // The CTA's r-th unit: rounds of gridDim.x consecutive units, taken left to right
  // in even rounds and right to left in odd ones (boustrophedon), so the heavy and
  // light query tiles of neighbouring units even out over a CTA's rounds (a plain
  // stride gives one CTA only heavy tiles when gridDim.x is a multiple of n_q_tiles
  // / 2, e.g. 148 CTAs over 8 tiles per slice: 30% idle at the tail).
  auto unit_of = [&](int round) {
    const int c = (round & 1) ? (int)gridDim.x - 1 - (int)blockIdx.x : (int)blockIdx.x;
    return round * (int)gridDim.x + c;
  };
  auto unit_tile = [&](int u, int& qt, int& sl, int& nkb) {
    sl = u / p.n_q_tiles;
    qt = p.n_q_tiles - 1 - (u - sl * p.n_q_tiles);
    int last_key = p.sk - 1;
    if (p.causal) last_key = min(last_key, qt * 128 + 127 + diag_shift);
    nkb = last_key < 0 ? 0 : last_key / 64 + 1;
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    *abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * D);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_launch_dependents();  // every CTA holds its TMEM before the next kernel is scheduled
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tds);
      tma_prefetch_desc(&tk);
      int it = 0;
      bool ok = true;
      for (int rd = 0, u = unit_of(0); u < units && ok; u = unit_of(++rd)) {
        int qt, sl, nkb;
        unit_tile(u, qt, sl, nkb);
        const int bh = p.bh0 + sl;
        const int hh = bh % p.nh, bb = bh / p.nh;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int st = it % STAGES;
          if (!mbar_wait(&empty[st], ((it / STAGES) & 1) ^ 1, abort, 40)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + st * L::kStageBytes;
          uint8_t* sb = sa + L::kABytes;
          mbar_arrive_expect_tx(&full[st], L::kStageBytes);
          // two consecutive 64-query blocks of key block kb: 16 KiB contiguous
          tma_load_4d(sa, &tds, &full[st], 0, 0, qt * 2, sl * nkb_all + kb);
#pragma unroll
          for (int c = 0; c < D / 64; ++c) tma_load_4d(sb + c * 8192, &tk, &full[st], c * 64, kb * 64, hh, bb);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_f16(128, D, BF16, true, true);
      const uint32_t s0 = smem_u32(smem);
      const uint64_t da_base = make_sdesc(s0, 8192, 1024);
      const uint64_t db_base = make_sdesc(s0 + L::kABytes, 8192, 1024);
      int it = 0, local = 0;
      bool ok = true;
      for (int rd = 0, u = unit_of(0); u < units && ok; u = unit_of(++rd), ++local) {
        int qt, sl, nkb;
        unit_tile(u, qt, sl, nkb);
        const int buf = local & 1;
        if (!mbar_wait(&acc_empty[buf], ((local >> 1) & 1) ^ 1, abort, 41)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + buf * D;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int st = it % STAGES;
          if (!mbar_wait(&full[st], (it / STAGES) & 1, abort, 42)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = sdesc_at(da_base, st * L::kStageBytes);
          const uint64_t db = sdesc_at(db_base, st * L::kStageBytes);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            tc_mma_f16_ss(d_tmem, sdesc_at(da, kk * 2048), sdesc_at(db, kk * 2048), idesc,
                          (kb | kk) != 0 ? 1u : 0u);
          tc_commit(&empty[st]);
        }
        tc_commit(&acc_full[buf]);
      }
    }
  } else {
    const int q = warp & 3;
    const int r = q * 32 + lane;
    int local = 0;
    for (int rd = 0, u = unit_of(0); u < units; u = unit_of(++rd), ++local) {
      int qt, sl, nkb;
      unit_tile(u, qt, sl, nkb);
      const int buf = local & 1;
      if (!mbar_wait(&acc_full[buf], (local >> 1) & 1, abort, 43)) break;
      tc_fence_after();
      const int qrow = qt * 128 + r;
      const uint32_t src = tmem + ((uint32_t)(q * 32) << 16) + buf * D;
      T* out = reinterpret_cast<T*>(p.dq) + p.ldq.row(p.bh0 + sl, qrow);
#pragma unroll 1
      for (int c0 = 0; c0 < D; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(src + c0, v);
        tmem_wait_ld();
        if (qrow < p.sq) {
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            const float* f = reinterpret_cast<const float*>(&v[e]);
            const float m = p.scale;
            uint4 w;
            w.x = BF16 ? pack_bf16x2(f[0] * m, f[1] * m) : pack_f16x2(f[0] * m, f[1] * m);
            w.y = BF16 ? pack_bf16x2(f[2] * m, f[3] * m) : pack_f16x2(f[2] * m, f[3] * m);
            w.z = BF16 ? pack_bf16x2(f[4] * m, f[5] * m) : pack_f16x2(f[4] * m, f[5] * m);
            w.w = BF16 ? pack_bf16x2(f[6] * m, f[7] * m) : pack_f16x2(f[6] * m, f[7] * m);
            *reinterpret_cast<uint4*>(out + c0 + e) = w;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * D);
  }
}

// ===========================================================================
// Fused backward: dK/dV units and dQ-from-dS units in one persistent kernel
// ===========================================================================
//
// The dK/dV work (one unit per (slice, 128-key tile), flash_attention.py:197-221)
// and the dQ work (one unit per (slice, 128-query tile): dQ = scale * dS K, the
// one tensor-core product that replaces the reference's second recompute,
// :224-243) run as units of ONE persistent launch, so every dS tile is read back
// while it is still in L2 and then dropped from L2 unwritten (discard.global.L2):
// the dS round trip through HBM of the two-kernel path -- a write and a read of
// 2 bytes per causal score, 34 GB per step at b8 h32 s8192 -- disappears, and with
// it most of the energy that held the power-capped clock down.
//
// * A dK/dV unit walks its query tiles from the LAST to the first, so all units
//   of a slice, which start close together, finish query tile i at about the
//   same time, high tiles first.  Its eight elementwise warps hand each dS^T
//   tile to a store warp (warp 10) through the shared staging tile; the store
//   warp issues the TMA stores and, once they have completed (bulk wait_group,
//   proxy fence), adds one to the query tile's counter (acquire-release).  The
//   add that completes the count publishes the dQ unit of that tile in a ready
//   queue.  The waits for store completion and the gpu-scope atomics stay off
//   the elementwise and MMA warps' path.
// * A dQ unit is handed out only once published, so a CTA never waits inside a
//   unit for another CTA.  It streams the tile's dS^T blocks and the slice's K
//   tiles through a ring (same MMA as attn_dq_ds_kernel), writes dQ, discards
//   the dS lines it read and counts the slice's finished dQ units.
// * Scheduling (thread 0, state in the workspace, zeroed per launch): a CTA takes
//   a published dQ unit if there is one, else the next dK/dV unit in slice-major,
//   heaviest-first order.  dS lives in `slots` slice-sized slots; slice s may
//   start once every dQ unit of slice s - slots has finished (its slot is free).
//   Every wait across CTAs happens in this claim loop, on work that was claimed
//   earlier and is running, so there is no cycle; the loop is bounded by
//   kWaitLimitNs and a global abort word stops every CTA after a timeout.
// Numerics are those of the two-kernel path (same dS values, same products, same
// summation order); no atomics touch any result.

constexpr int kFusedMaxDqStages = 6;
// Warps: 0 TMA loads, 1 TMEM + MMA, 2 .. 2 + EW - 1 elementwise (dK/dV units) / dQ
// epilogue (dQ units), then one warp of dS stores + signals, then the scheduler warp,
// which claims the CTA's next unit while the current one runs (at short sequences a
// dK/dV unit is only a few tiles, and a claim is several gpu-scope atomics).  EW = 8
// (two warps per TMEM lane quadrant, 64 query columns each; up to 168 registers a
// thread) or 16 (four per quadrant, 32 columns each; more warps per scheduler but
// ~100 registers).
template <int EW>
constexpr int fused_threads() { return 32 * (EW + 4); }
enum { kSchedNext = 0, kSchedHead = 1, kSchedTail = 2, kSchedAbort = 3, kSchedInts = 8 };

struct FusedParams {
  int nq, nkt;       // query tiles / key tiles (128 rows each) per slice
  int n_slices;      // slices bh0 .. bh0 + n_slices - 1
  int slots;         // dS slots (slice-sized)
  int* sched;        // kSchedInts ints
  int* ready;        // [n_slices * nq / 2] published dQ unit ids (-1 = not yet written)
  int* row_cnt;      // [n_slices * nq / 2] dS tile signals per dQ unit
  int* dq_done;      // [n_slices] finished dQ units per slice
  uint8_t* ds;       // slot 0 of the dS blocks
  int64_t ds_slot_bytes;
  void* dq;
  Bhsd ldq;
};

template <int D>
struct FusedSmem {
  using W = WideSmem<D>;
  static constexpr int kDataBytes = W::kDataBytes;
  static constexpr int kDqABytes = 128 * 64 * 2;  // dS^T of one query tile: 2 boxes of 64 queries x 64 keys
  static constexpr int kDqBBytes = 64 * D * 2;    // K: D/64 boxes of 64 d x 64 keys
  static constexpr int kDqStageBytes = 2 * kDqABytes + kDqBBytes;  // two query tiles share the K block
  static constexpr int kDqStages =
      kDataBytes / kDqStageBytes < kFusedMaxDqStages ? kDataBytes / kDqStageBytes : kFusedMaxDqStages;
  static_assert(kDqStages >= 2, "dQ ring needs two stages");
  static constexpr int kNumDkvBars = W::kNumBars + 2;  // + stg_full, stg_free
  static constexpr int kNumDqBars = 2 * kDqStages + 1;
  // barriers, then TMEM slot, local abort, unit, kind, set-initialised flags
  // + TMEM slot and the CTA's scheduling words (32 bytes), per-warp store progress (32)
  static constexpr int kBarBytes = (kNumDkvBars + kNumDqBars) * 8 + 64;
  static_assert(kBarBytes <= 512, "barrier block must fit the alignment slack rule");
  // Data at the first 1024-byte boundary; the barrier block in the slack before it
  // when that holds 512 bytes, else right after the data (slack < 512 then).
  static constexpr int kTotal = kDataBytes + 1024;
};

// A dQ unit covers the query tiles 2 u and 2 u + 1 of a slice (they share every K
// block it loads).  Signals it waits for: one per key tile per query tile.
__device__ __forceinline__ int fused_producers(const FusedParams& fp, int causal, int pair) {
  const int q0 = 2 * pair, q1 = 2 * pair + 1;
  return causal ? min(q0 + 1, fp.nkt) + min(q1 + 1, fp.nkt) : 2 * fp.nkt;
}

// Claim the next unit (thread 0 only).  Returns the unit id and sets kind (0 dK/dV,
// 1 dQ), or -1 when every unit has been handed out or the launch aborted.
// dQ units first: a CTA takes the oldest published one (compare-and-swap on the
// queue head, retried with the value it returns).  Otherwise it draws a dK/dV
// ticket with fetch-and-add (no retries however many CTAs draw at once) and keeps
// it in `pending` until the ticket's dS slot is free, serving dQ units
// meanwhile.  A ticket of slice s waits only for the dQ units of slice
// s - slots, which depend only on dK/dV tickets drawn before it, so the oldest
// waiting ticket can always start: no cycle.
__device__ __noinline__ int fused_claim(const FusedParams& fp, int& kind, int& pending) {
  int* s = fp.sched;
  const int n_dkv = fp.n_slices * fp.nkt;
  const int n_dq = fp.n_slices * (fp.nq / 2);
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if ((spins & 15u) == 0 && ld_relaxed_gpu(&s[kSchedAbort])) return -1;
    int h = ld_relaxed_gpu(&s[kSchedHead]);
    const int t = ld_relaxed_gpu(&s[kSchedTail]);
    while (h < t) {
      const int old = atom_cas_gpu(&s[kSchedHead], h, h + 1);
      if (old == h) {
        int v;
        while ((v = ld_acquire_gpu(&fp.ready[h])) < 0) {  // the publisher is between its two writes
          if ((++spins & 63u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) {
            report_timeout(61);
            st_relaxed_gpu(&s[kSchedAbort], 1);
            return -1;
          }
        }
        kind = 1;
        return v;
      }
      h = old;
    }
    if (h >= n_dq) return -1;  // every dQ unit handed out: every dK/dV unit ran
    if (pending < 0) pending = atomicAdd(&s[kSchedNext], 1);
    if (pending < n_dkv) {
      const int sl = pending / fp.nkt;
      if (sl < fp.slots || ld_acquire_gpu(&fp.dq_done[sl - fp.slots]) >= fp.nq / 2) {
        const int u = pending;
        pending = -1;
        kind = 0;
        return u;
      }
    }
    __nanosleep(200);
    if ((++spins & 63u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) {
      report_timeout(60);
      st_relaxed_gpu(&s[kSchedAbort], 1);
      return -1;
    }
  }
}

// Signal that the dS^T tile of one key tile for query tile `qt` of slice `sl` is in
// global memory (the store warp, after the TMA stores of that tile completed).
__device__ __forceinline__ void fused_signal(const FusedParams& fp, int causal, int sl, int qt) {
  fence_proxy_async_global();
  const int id = sl * (fp.nq / 2) + (qt >> 1);
  const int old = atom_add_acq_rel_gpu(&fp.row_cnt[id], 1);
  if (old + 1 == fused_producers(fp, causal, qt >> 1)) {
    const int slot = atomicAdd(&fp.sched[kSchedTail], 1);
    st_release_gpu(&fp.ready[slot], id);
  }
}

template <int D, bool BF16, int EW>
__global__ void __launch_bounds__(fused_threads<EW>(), 1)
    attn_bwd_fused_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                          const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tdo,
                          const __grid_constant__ CUtensorMap tlse, const __grid_constant__ CUtensorMap tdelta,
                          const __grid_constant__ CUtensorMap tds_st, const __grid_constant__ CUtensorMap tds_ld,
                          const __grid_constant__ CUtensorMap tk64, const BwdParams p, const FusedParams fp) {
  using W = WideSmem<D>;
  using L = FusedSmem<D>;
  constexpr int S = W::kStages;
  constexpr int QS = L::kDqStages;
  constexpr int kStoreWarp = 2 + EW;
  constexpr int CW = 128 * 4 / EW;  // query columns per elementwise warp (64 or 32)
  constexpr int NG = EW / 4;        // elementwise warps per TMEM lane quadrant
  // With 64 query columns a warp owns one whole 32-key x 64-query block of the dS^T
  // staging tile: it stores the block itself (one TMA store) and, once that store has
  // completed, publishes its progress; the store warp signals a tile to the dQ units
  // when every warp's progress has passed it.  No warp waits for the others' staging
  // writes.  With 32 columns two warps share a block and the store warp stores the
  // whole tile.
  constexpr bool kWarpStores = CW == 64;
  typedef typename std::conditional<BF16, __nv_bfloat16, __half>::type T;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem - smem_raw >= 512 ? smem_raw : smem + L::kDataBytes);
  // dK/dV unit barriers (as in attn_dkv_wide_kernel)
  uint64_t* x_full = bars + 0;
  uint64_t* y_full = bars + 1;
  uint64_t* y_empty = bars + 1 + S;
  uint64_t* s_full = bars + 1 + 2 * S;
  uint64_t* dp_full = s_full + 1;
  uint64_t* p_full = s_full + 2;
  uint64_t* dp_free = s_full + 3;
  uint64_t* ds_full = s_full + 4;
  uint64_t* acc_full = s_full + 5;
  uint64_t* p_half = s_full + 6;
  uint64_t* stg_full = s_full + 7;  // the eight elementwise warps wrote the dS^T staging tile
  uint64_t* stg_free = s_full + 8;  // the store warp's TMA stores have read it
  // dQ unit barriers
  uint64_t* q_full = bars + L::kNumDkvBars;
  uint64_t* q_empty = q_full + QS;
  uint64_t* q_acc = q_full + 2 * QS;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::kNumDkvBars + L::kNumDqBars);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* s_unit = abort + 1;
  volatile int* s_kind = abort + 2;
  volatile int* s_inited = abort + 3;  // bit 0: dK/dV set, bit 1: dQ set
  volatile int* s_next = abort + 4;    // the scheduler warp's claim for the next unit
  volatile int* s_next_kind = abort + 5;
  // Work the current unit's MMA lane has not issued yet (query tiles of a dK/dV unit,
  // key blocks of a dQ unit); 0 once its MMAs have completed, when the scheduler claims
  // the next unit.
  volatile int* s_left = abort + 6;
  // kWarpStores: tiles of the current dK/dV unit whose dS store has completed, per
  // elementwise warp (monotonic counters: the store warp may fall any number of tiles
  // behind without missing one, which an mbarrier phase could not guarantee)
  int* s_prog = const_cast<int*>(abort + 7);
  constexpr int kSchedWarp = 3 + EW;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int diag_shift = p.sk - p.sq;
  const int nkb_all = p.sk / 64;

  if (threadIdx.x == 0) {
    *abort = 0;
    *s_inited = 0;
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_launch_dependents();
  pdl_wait();
  const uint32_t t_dv = tmem + 256;
  const uint32_t t_dk = tmem + 256 + D;

  int pending = -1;  // scheduler lane: a dK/dV ticket whose dS slot is not free yet
  // The scheduler warp's lane 0 makes every claim: the first one here, each next one
  // once the current unit's MMAs have completed (below).
  auto claim_next = [&]() {
    int kind = 0;
    const int u = *abort ? -1 : fused_claim(fp, kind, pending);
    *s_next = u;
    *s_next_kind = kind;
  };
  if (warp == kSchedWarp && lane == 0) claim_next();
  __syncthreads();
  while (true) {
    // ---------------------------------------------------------------- next unit
    if (threadIdx.x == 0) {
      const int kind = *s_next_kind;
      const int u = *abort ? -1 : *s_next;
      *s_unit = u;
      *s_kind = kind;
      *s_left = 0x7fffffff;
      if (u >= 0) {
        fence_proxy_async_global();  // TMA traffic of this unit after the acquire of its inputs / slot
        const int bit = kind ? 2 : 1;
        if (kind == 0) {
          if (*s_inited & 1) {
            for (int i = 0; i < L::kNumDkvBars; ++i) mbar_inval(&bars[i]);
          }
          mbar_init(x_full, 1);
          for (int i = 0; i < S; ++i) {
            mbar_init(&y_full[i], 1);
            mbar_init(&y_empty[i], 1);
          }
          mbar_init(s_full, 1);
          mbar_init(dp_full, 1);
          mbar_init(p_full, 8);  // one arrival per 32-query chunk 1, 3 (four lane quadrants each)
          mbar_init(p_half, 8);  // one arrival per 32-query chunk 0, 2
          mbar_init(dp_free, EW);
          mbar_init(ds_full, EW);
          mbar_init(acc_full, 1);
          mbar_init(stg_full, EW);
          mbar_init(stg_free, 1);
          if constexpr (kWarpStores)
            for (int w = 0; w < EW; ++w) s_prog[w] = 0;
        } else {
          if (*s_inited & 2) {
            for (int i = 0; i < L::kNumDqBars; ++i) mbar_inval(&q_full[i]);
          }
          for (int i = 0; i < QS; ++i) {
            mbar_init(&q_full[i], 1);
            mbar_init(&q_empty[i], 1);
          }
          mbar_init(q_acc, 1);
        }
        *s_inited = *s_inited | bit;
        fence_mbar_init();
      }
    }
    __syncthreads();
    const int unit = *s_unit;
    if (unit < 0) break;

    if (warp == kSchedWarp) {
      if (lane == 0) {
        // Claim once this unit's MMAs have completed: the claim (several gpu-scope
        // atomics) overlaps the unit's epilogue, and the claimed unit starts right after.
        // Claiming earlier (two query tiles before the end) delayed the claimed dQ units
        // by those tiles: their dS was read back later, and ~1/3 more DRAM traffic.
        const uint64_t t0 = globaltimer_ns();
        uint32_t spins = 0;
        while (*s_left > 0 && !*abort) {
          __nanosleep(128);
          if ((++spins & 63u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) {
            report_timeout(65);
            *abort = 1;
          }
        }
        claim_next();  // s_next is read by thread 0 after the unit-end barrier
        const int nu = *s_next;
        if (nu >= 0 && *s_next_kind == 0) {
          // warm L2 with the next dK/dV unit's K, V and first (last-index) Q, dO tiles
          const int nsl = nu / fp.nkt;
          const int nbh = p.bh0 + nsl;
          const int nhh = nbh % p.l0.nh, nbb = nbh / p.l0.nh;
          const int nx0 = (nu - nsl * fp.nkt) * BX;
          const int ny = ((p.sq + kWideY - 1) / kWideY - 1) * kWideY;
#pragma unroll
          for (int c = 0; c < W::kChunks; ++c) {
            tma_prefetch_4d(&tk, c * 64, nx0, nhh, nbb);
            tma_prefetch_4d(&tv, c * 64, nx0, nhh, nbb);
            tma_prefetch_4d(&tq, c * 64, ny, nhh, nbb);
            tma_prefetch_4d(&tdo, c * 64, ny, nhh, nbb);
          }
        }
      }
    } else if (*s_kind == 0) {
      // ============================================================ dK/dV unit
      const int sl = unit / fp.nkt;
      const int ktile = unit - sl * fp.nkt;
      const int slot = sl % fp.slots;
      const int bh = p.bh0 + sl;
      const int hh = bh % p.l0.nh, bb = bh / p.l0.nh;
      const int x0 = ktile * BX;
      int j0 = 0;
      const int j1 = (p.sq + kWideY - 1) / kWideY;
      if (p.causal) j0 = max(0, x0 - diag_shift) / kWideY;
      const int n_y = max(0, j1 - j0);
      // query tile of the i-th step: last tile first
      auto ytile = [&](int i) { return j1 - 1 - i; };
      auto load_y = [&](int i) {
        const int s = i % S;
        uint8_t* y1 = smem + W::kYOff + s * W::kStageBytes;
        uint8_t* y2 = y1 + W::kYBytes;
        mbar_arrive_expect_tx(&y_full[s], 2 * W::kYBytes + 2 * kWideY * 4);
        const int yrow = ytile(i) * kWideY;
#pragma unroll
        for (int c = 0; c < W::kChunks; ++c) {
          tma_load_4d(y1 + c * (kWideY * 128), &tq, &y_full[s], c * 64, yrow, hh, bb);
          tma_load_4d(y2 + c * (kWideY * 128), &tdo, &y_full[s], c * 64, yrow, hh, bb);
        }
        float* st = reinterpret_cast<float*>(y2 + W::kYBytes);
        tma_load_2d(st, &tlse, &y_full[s], yrow, bh);
        tma_load_2d(st + kWideY, &tdelta, &y_full[s], yrow, bh);
      };
      const int n_pre = min(n_y, S);
      if (threadIdx.x == 0 && n_y > 0) {
        mbar_arrive_expect_tx(x_full, 2 * W::kXBytes);
#pragma unroll
        for (int c = 0; c < W::kChunks; ++c) {
          tma_load_4d(smem + W::kX1Off + c * (BX * 128), &tk, x_full, c * 64, x0, hh, bb);
          tma_load_4d(smem + W::kX2Off + c * (BX * 128), &tv, x_full, c * 64, x0, hh, bb);
        }
        for (int i = 0; i < n_pre; ++i) load_y(i);
      }
      if (warp == 0) {
        if (lane == 0 && n_y > 0) {
          for (int i = n_pre; i < n_y; ++i) {
            if (!mbar_wait(&y_empty[i % S], ((i / S) & 1) ^ 1, abort, 41)) break;
            load_y(i);
          }
        }
      } else if (warp == 1) {
        if (lane == 0 && n_y > 0) {
          constexpr uint32_t idesc_t = make_idesc_f16(BX, kWideY, BF16, false, false);
          constexpr uint32_t idesc_a = make_idesc_f16(BX, D, BF16, false, true);
          const uint64_t dx1 = make_sdesc(smem_u32(smem + W::kX1Off), 16, 1024);
          const uint64_t dx2 = make_sdesc(smem_u32(smem + W::kX2Off), 16, 1024);
          const uint64_t dy_k = make_sdesc(smem_u32(smem + W::kYOff), 16, 1024);
          const uint64_t dy_mn = make_sdesc(smem_u32(smem + W::kYOff), kWideY * 128, 1024);
          bool ok = mbar_wait(x_full, 0, abort, 42);
          auto region = [&](int i, bool is_s) -> uint32_t { return (((i & 1) ^ (is_s ? 0 : 1)) ? 128u : 0u); };
          auto issue_prod = [&](int i, bool is_s) {
            const uint64_t dy = sdesc_at(dy_k, (i % S) * W::kStageBytes + (is_s ? 0 : W::kYBytes));
            const uint64_t dx = is_s ? dx1 : dx2;
            const uint32_t dst = tmem + region(i, is_s);
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint32_t xo = (kk >> 2) * (BX * 128) + (kk & 3) * 32;
              const uint32_t yo = (kk >> 2) * (kWideY * 128) + (kk & 3) * 32;
              tc_mma_f16_ss(dst, sdesc_at(dx, xo), sdesc_at(dy, yo), idesc_t, kk != 0);
            }
            tc_commit(is_s ? s_full : dp_full);
          };
          // Query step kk (queries 16 kk .. 16 kk + 15) belongs to elementwise column
          // group 16 kk / CW, which packs P^T into the first CW / 2 columns of its own
          // CW and dS^T into the last CW / 2: P^T of step kk at CW g + (16 kk % CW) / 2,
          // dS^T CW / 2 further.
          auto packed = [](int kk) -> uint32_t { return (uint32_t)(CW * (16 * kk / CW) + (16 * kk % CW) / 2); };
          auto issue_dv = [&](int i, int part) {
            const uint64_t dm2 = sdesc_at(dy_mn, (i % S) * W::kStageBytes + W::kYBytes);
            const uint32_t pa = tmem + region(i, true);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int kk = (q >> 1) * 4 + part * 2 + (q & 1);  // part 0: groups 0, 2; part 1: groups 1, 3
              tc_mma_f16_ts(t_dv, pa + packed(kk), sdesc_at(dm2, kk * 2048), idesc_a, (i > 0 || kk > 0) ? 1u : 0u);
            }
          };
          auto issue_dk = [&](int i) {
            const uint64_t dm1 = sdesc_at(dy_mn, (i % S) * W::kStageBytes);
            const uint32_t da = tmem + region(i, true) + CW / 2;
#pragma unroll
            for (int kk = 0; kk < kWideY / 16; ++kk)
              tc_mma_f16_ts(t_dk, da + packed(kk), sdesc_at(dm1, kk * 2048), idesc_a, (i > 0 || kk > 0) ? 1u : 0u);
            tc_commit(&y_empty[i % S]);
          };
          if (ok && (ok = mbar_wait(&y_full[0], 0, abort, 43))) {
            tc_fence_after();
            issue_prod(0, true);
            issue_prod(0, false);
          }
          for (int i = 0; ok && i < n_y; ++i) {
            const bool more = i + 1 < n_y;
            *s_left = n_y - i;
            if (!(ok = mbar_wait(p_half, i & 1, abort, 52))) break;
            tc_fence_after();
            issue_dv(i, 0);
            if (!(ok = mbar_wait(p_full, i & 1, abort, 45))) break;
            if (more) {
              if (!(ok = mbar_wait(dp_free, i & 1, abort, 44))) break;
              if (!(ok = mbar_wait(&y_full[(i + 1) % S], ((i + 1) / S) & 1, abort, 43))) break;
            }
            tc_fence_after();
            if (more) issue_prod(i + 1, true);
            issue_dv(i, 1);
            if (!(ok = mbar_wait(ds_full, i & 1, abort, 46))) break;
            tc_fence_after();
            issue_dk(i);
            if (more) issue_prod(i + 1, false);
          }
          tc_commit(acc_full);
          mbar_drain(acc_full, 0);
        }
        if (lane == 0) *s_left = 0;
      } else if (warp == kStoreWarp) {
        // ------------------------------------------------ dS^T stores + signals
        // kWarpStores: the elementwise warps store their own blocks; this warp signals
        // each tile once every warp's progress counter has passed it.  Otherwise this
        // warp issues one TMA store per 32-key x 64-query staging block; the stg_free
        // arrival lets the elementwise warps write the next tile while the stores drain
        // to L2; a tile's query tile is signalled once its stores have completed (one
        // tile later, so the wait is off every other warp's path).
        if (kWarpStores && lane == 0) {
          const uint64_t t0 = globaltimer_ns();
          uint32_t spins = 0;
          for (int i = 0; i < n_y && !*abort; ++i) {
            // every warp's store of tile i has completed
            while (true) {
              int lo = n_y;
#pragma unroll
              for (int w = 0; w < EW; ++w) lo = min(lo, ld_acquire_cta_shared(&s_prog[w]));
              if (lo > i || *abort) break;
              if ((++spins & 63u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) {
                report_timeout(55);
                *abort = 1;
              }
            }
            if (*abort) break;
            fused_signal(fp, p.causal, sl, ytile(i));
          }
        } else if (lane == 0) {
          bool ok = true;
          int prev_qt = -1;
          const uint64_t keep = l2_policy_evict_last();  // read back soon by a dQ unit
          for (int i = 0; i < n_y; ++i) {
            if (!mbar_wait(stg_full, i & 1, abort, 54)) {
              ok = false;
              break;
            }
            const int y0 = ytile(i) * kWideY;
#pragma unroll
            for (int hq = 0; hq < 8; ++hq) {
              const int hb = hq >> 2, qw = hq & 3;
              const int key = x0 + qw * 32;
              tma_store_4d_hint(&tds_st, smem + W::kStgOff + hb * (BX * 128) + qw * 4096, 0, key & 63,
                                (y0 >> 6) + hb, slot * nkb_all + (key >> 6), keep);
            }
            bulk_commit_group();
            bulk_wait_group_read0();
            mbar_arrive(stg_free);
            if (prev_qt >= 0) {
              bulk_wait_group1();
              fused_signal(fp, p.causal, sl, prev_qt);
            }
            prev_qt = y0 / kWideY;
          }
          bulk_wait_group0();
          if (ok && prev_qt >= 0) fused_signal(fp, p.causal, sl, prev_qt);
        }
      } else {
        // ------------------------------------------------ elementwise warps
        // warp w: TMEM lane quadrant w % 4 (key rows), query columns [CW cq, CW cq + CW)
        // of each tile, cq = (w - 2) / 4; a warp reads and rewrites only its own CW
        // columns of the S^T region (P^T packed into the first CW / 2, dS^T the rest)
        const int qw = warp & 3;
        const int cq = (warp - 2) >> 2;
        const int r = qw * 32 + lane;
        const int xrow = x0 + r;
        const uint32_t lane_off = (uint32_t)(qw * 32) << 16;
        const uint32_t t_col = tmem + lane_off + CW * cq;
        // staging tile: [64-query half][128 keys][128 B swizzled]; this warp's 2 CW bytes of each row
        uint8_t* stg = smem + W::kStgOff + (CW * cq / 64) * (BX * 128) + qw * 4096;
        const int g0 = (CW * cq % 64) / 8;  // first 16-byte granule of the row
        bool ok = true;
        for (int i = 0; ok && i < n_y; ++i) {
          const int ph = i & 1;
          const int y0 = ytile(i) * kWideY;
          const int s = i % S;
          const uint32_t t_s = t_col + ((i & 1) ? 128u : 0u);
          const uint32_t t_dp = t_col + ((i & 1) ? 0u : 128u);
          const bool need_mask = (y0 + kWideY > p.sq) || (p.causal && x0 + BX - 1 > y0 + diag_shift);
          if (!mbar_wait(s_full, ph, abort, 47) || !mbar_wait(&y_full[s], (i / S) & 1, abort, 48)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const float* st = reinterpret_cast<const float*>(smem + W::kYOff + s * W::kStageBytes + 2 * W::kYBytes) + CW * cq;
          uint32_t pf[CW];
#pragma unroll
          for (int c = 0; c < CW; c += 32) tmem_ld32(t_s + c, *reinterpret_cast<uint32_t(*)[32]>(&pf[c]));
          tmem_wait_ld();
          {
            // four columns per step: one 16-byte load of lse, packed f32x2 math
            // (each lane rounds exactly like fmaf(s, scale*log2e, -(lse*log2e)))
            const uint64_t sc2 = f2_make(p.scale_log2, p.scale_log2);
            const uint64_t nlog2e2 = f2_make(-kLog2e, -kLog2e);
            // 32-query chunks: P of chunk j is packed, published (p_half for even
            // global chunks, p_full for odd) and dV's query steps on it can start
            auto chunk_a = [&](auto c0) {
              constexpr int C0 = decltype(c0)::value;
              auto body = [&](auto masked) {
#pragma unroll
                for (int c = C0; c < C0 + 32; c += 4) {
                  const float4 l4 = *reinterpret_cast<const float4*>(st + c);
                  const uint64_t x01 = f2_fma(f2_make_bits(pf[c], pf[c + 1]), sc2, f2_mul(f2_make(l4.x, l4.y), nlog2e2));
                  const uint64_t x23 = f2_fma(f2_make_bits(pf[c + 2], pf[c + 3]), sc2, f2_mul(f2_make(l4.z, l4.w), nlog2e2));
                  float x[4] = {f2_lo(x01), f2_hi(x01), f2_lo(x23), f2_hi(x23)};
                  if constexpr (decltype(masked)::value) {
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                      const int qry = y0 + CW * cq + c + u;
                      const bool valid = qry < p.sq && !(p.causal && xrow > qry + diag_shift);
                      x[u] = valid ? x[u] : -INFINITY;
                    }
                  }
#pragma unroll
                  for (int u = 0; u < 4; ++u) pf[c + u] = __float_as_uint(ex2_approx(x[u]));
                }
              };
              if (need_mask)
                body(std::true_type{});
              else
                body(std::false_type{});
              uint32_t pp[16];
#pragma unroll
              for (int c = 0; c < 32; c += 2) {
                const float a0 = __uint_as_float(pf[C0 + c]), a1 = __uint_as_float(pf[C0 + c + 1]);
                pp[c / 2] = BF16 ? pack_bf16x2(a0, a1) : pack_f16x2(a0, a1);
              }
              tmem_st16(t_s + C0 / 2, pp);
              tmem_wait_st();
              tc_fence_before();
              __syncwarp();
              const int chunk = (CW * cq + C0) / 32;
              if (lane == 0) mbar_arrive((chunk & 1) ? p_full : p_half);
            };
            chunk_a(std::integral_constant<int, 0>{});
            if constexpr (CW == 64) chunk_a(std::integral_constant<int, 32>{});
          }
          if (!mbar_wait(dp_full, ph, abort, 49)) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint32_t b[CW];
#pragma unroll
          for (int c = 0; c < CW; c += 32) tmem_ld32(t_dp + c, *reinterpret_cast<uint32_t(*)[32]>(&b[c]));
          tmem_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(dp_free);
          if constexpr (kWarpStores) {
            // this warp's own store of the previous tile has read its staging block
            if (lane == 0) bulk_wait_group_read0();
            __syncwarp();
          } else if (i > 0 && !mbar_wait(stg_free, (i - 1) & 1, abort, 53)) {
            // the store warp's TMA stores of the previous tile have read the staging tile
            ok = false;
            break;
          }
          uint8_t* row = stg + lane * 128;
#pragma unroll
          for (int hb = 0; hb < CW / 16; ++hb) {  // 16 columns at a time (fewer live registers)
            uint32_t dd[8];
#pragma unroll
            for (int e = 0; e < 16; e += 4) {
              const int c = hb * 16 + e;
              const float4 d4 = *reinterpret_cast<const float4*>(st + kWideY + c);
              const uint64_t d01 = f2_mul(f2_make_bits(pf[c], pf[c + 1]),
                                          f2_sub(f2_make_bits(b[c], b[c + 1]), f2_make(d4.x, d4.y)));
              const uint64_t d23 = f2_mul(f2_make_bits(pf[c + 2], pf[c + 3]),
                                          f2_sub(f2_make_bits(b[c + 2], b[c + 3]), f2_make(d4.z, d4.w)));
              dd[e / 2] = BF16 ? pack_bf16x2(f2_lo(d01), f2_hi(d01)) : pack_f16x2(f2_lo(d01), f2_hi(d01));
              dd[e / 2 + 1] = BF16 ? pack_bf16x2(f2_lo(d23), f2_hi(d23)) : pack_f16x2(f2_lo(d23), f2_hi(d23));
            }
            tmem_st8(t_s + CW / 2 + 8 * hb, dd);
#pragma unroll
            for (int v = 0; v < 2; ++v) {
              const int g16 = g0 + 2 * hb + v;
              *reinterpret_cast<uint4*>(row + ((g16 ^ (lane & 7)) << 4)) =
                  make_uint4(dd[4 * v], dd[4 * v + 1], dd[4 * v + 2], dd[4 * v + 3]);
            }
          }
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(ds_full);
          fence_proxy_async_smem();  // the staging writes, before the TMA store reads them
          __syncwarp();
          if constexpr (kWarpStores) {
            if (lane == 0) {
              const int key = x0 + qw * 32;
              // evict_last: dS^T is read back soon by a dQ unit
              tma_store_4d_hint(&tds_st, stg, 0, key & 63, (y0 + CW * cq) >> 6, slot * nkb_all + (key >> 6),
                                l2_policy_evict_last());
              bulk_commit_group();
              if (i > 0) {  // the previous tile's store has completed
                bulk_wait_group1();
                st_release_cta_shared(&s_prog[warp - 2], i);
              }
            }
          } else if (lane == 0) {
            mbar_arrive(stg_full);
          }
        }
        if constexpr (kWarpStores) {
          if (lane == 0) {
            bulk_wait_group0();  // complete before the unit ends (the next unit reuses the smem)
            if (ok) st_release_cta_shared(&s_prog[warp - 2], n_y);
          }
          __syncwarp();
        }
        // epilogue: the first NG / 2 column groups store dK (x scale), the others dV,
        // D / (NG / 2) columns each
        constexpr int OC = D / (NG / 2);
        const int hk = cq / (NG / 2), c_begin = (cq % (NG / 2)) * OC;
        if (n_y > 0 && ok && mbar_wait(acc_full, 0, abort, 51)) {
          tc_fence_after();
          const bool row_ok = xrow < p.sk;
          T* out = reinterpret_cast<T*>(hk == 0 ? p.out0 : p.out1) + (hk == 0 ? p.l0 : p.l1).row(bh, xrow);
          const uint32_t src = (hk == 0 ? t_dk : t_dv) + lane_off;
          const float mul = hk == 0 ? p.scale : 1.0f;
#pragma unroll
          for (int c0 = c_begin; c0 < c_begin + OC; c0 += 32) {
            uint32_t v[32];
            tmem_ld32(src + c0, v);
            tmem_wait_ld();
            if (row_ok) {
#pragma unroll
              for (int e = 0; e < 32; e += 8) {
                uint4 w;
                const float* f = reinterpret_cast<const float*>(&v[e]);
                w.x = BF16 ? pack_bf16x2(f[0] * mul, f[1] * mul) : pack_f16x2(f[0] * mul, f[1] * mul);
                w.y = BF16 ? pack_bf16x2(f[2] * mul, f[3] * mul) : pack_f16x2(f[2] * mul, f[3] * mul);
                w.z = BF16 ? pack_bf16x2(f[4] * mul, f[5] * mul) : pack_f16x2(f[4] * mul, f[5] * mul);
                w.w = BF16 ? pack_bf16x2(f[6] * mul, f[7] * mul) : pack_f16x2(f[6] * mul, f[7] * mul);
                *reinterpret_cast<uint4*>(out + c0 + e) = w;
              }
            }
          }
        } else if (n_y == 0 && xrow < p.sk) {
          T* out = reinterpret_cast<T*>(hk == 0 ? p.out0 : p.out1) + (hk == 0 ? p.l0 : p.l1).row(bh, xrow);
          for (int c = c_begin; c < c_begin + OC; ++c) out[c] = DT<T>::from_f(0.f);
        }
      }
    } else {
      // ============================================================ dQ unit
      // query tiles qt0 = 2 u' and qt0 + 1 of slice sl; K blocks up to the higher
      // tile's diagonal, the lower tile's MMAs stop at its own
      const int sl = unit / (fp.nq / 2);
      const int qt0 = 2 * (unit - sl * (fp.nq / 2));
      const int slot = sl % fp.slots;
      const int bh = p.bh0 + sl;
      const int hh = bh % p.l0.nh, bb = bh / p.l0.nh;
      auto kblocks = [&](int qt) {
        int last_key = p.sk - 1;
        if (p.causal) last_key = min(last_key, qt * 128 + 127 + diag_shift);
        return last_key < 0 ? 0 : last_key / 64 + 1;
      };
      const int nkb0 = kblocks(qt0), nkb = kblocks(qt0 + 1);
      const int nqb = (p.sq + 63) / 64;  // query blocks per key block in the dS layout
      if (warp == 0) {
        if (lane == 0) {
          const uint64_t last_use = l2_policy_evict_first();  // dS is read once, then discarded
          for (int kb = 0; kb < nkb; ++kb) {
            const int st = kb % QS;
            if (!mbar_wait(&q_empty[st], ((kb / QS) & 1) ^ 1, abort, 62)) break;
            uint8_t* sa = smem + st * L::kDqStageBytes;
            uint8_t* sb = sa + 2 * L::kDqABytes;
            const bool both = kb < nkb0;
            mbar_arrive_expect_tx(&q_full[st], (both ? 2 : 1) * L::kDqABytes + L::kDqBBytes);
            tma_load_4d_hint(sa + L::kDqABytes, &tds_ld, &q_full[st], 0, 0, (qt0 + 1) * 2, slot * nkb_all + kb, last_use);
            if (both) tma_load_4d_hint(sa, &tds_ld, &q_full[st], 0, 0, qt0 * 2, slot * nkb_all + kb, last_use);
#pragma unroll
            for (int c = 0; c < D / 64; ++c) tma_load_4d(sb + c * 8192, &tk64, &q_full[st], c * 64, kb * 64, hh, bb);
          }
        }
      } else if (warp == 1) {
        if (lane == 0) {
          constexpr uint32_t idesc = make_idesc_f16(128, D, BF16, true, true);
          const uint32_t s0 = smem_u32(smem);
          const uint64_t da_base = make_sdesc(s0, 8192, 1024);
          const uint64_t db_base = make_sdesc(s0 + 2 * L::kDqABytes, 8192, 1024);
          for (int kb = 0; kb < nkb; ++kb) {
            const int st = kb % QS;
            *s_left = nkb - kb;
            if (!mbar_wait(&q_full[st], (kb / QS) & 1, abort, 63)) break;
            tc_fence_after();
            const uint64_t da = sdesc_at(da_base, st * L::kDqStageBytes);
            const uint64_t db = sdesc_at(db_base, st * L::kDqStageBytes);
            // accumulators: tile qt0 at columns [0, D), qt0 + 1 at [D, 2 D)
            if (kb < nkb0) {
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)
                tc_mma_f16_ss(tmem, sdesc_at(da, kk * 2048), sdesc_at(db, kk * 2048), idesc, (kb | kk) != 0 ? 1u : 0u);
            }
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              tc_mma_f16_ss(tmem + D, sdesc_at(da, L::kDqABytes + kk * 2048), sdesc_at(db, kk * 2048), idesc,
                            (kb | kk) != 0 ? 1u : 0u);
            tc_commit(&q_empty[st]);
          }
          tc_commit(q_acc);
          mbar_drain(q_acc, 0);
        }
        if (lane == 0) *s_left = 0;
      } else if (warp < kStoreWarp) {
        // the first NG / 2 column groups store tile qt0's dQ, the others tile qt0 + 1,
        // D / (NG / 2) columns each
        constexpr int OC = D / (NG / 2);
        const int qw = warp & 3;
        const int cq = (warp - 2) >> 2;
        const int tile = cq / (NG / 2), c_begin = (cq % (NG / 2)) * OC;
        const int r = qw * 32 + lane;
        if (nkb > 0 && mbar_wait(q_acc, 0, abort, 64)) {
          tc_fence_after();
          const int qrow = (qt0 + tile) * 128 + r;
          const uint32_t src = tmem + ((uint32_t)(qw * 32) << 16) + tile * D;
          T* out = reinterpret_cast<T*>(fp.dq) + fp.ldq.row(bh, qrow);
          const float m = p.scale;
#pragma unroll
          for (int c0 = c_begin; c0 < c_begin + OC; c0 += 32) {
            uint32_t v[32];
            tmem_ld32(src + c0, v);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; e += 8) {
              const float* f = reinterpret_cast<const float*>(&v[e]);
              uint4 w;
              w.x = BF16 ? pack_bf16x2(f[0] * m, f[1] * m) : pack_f16x2(f[0] * m, f[1] * m);
              w.y = BF16 ? pack_bf16x2(f[2] * m, f[3] * m) : pack_f16x2(f[2] * m, f[3] * m);
              w.z = BF16 ? pack_bf16x2(f[4] * m, f[5] * m) : pack_f16x2(f[4] * m, f[5] * m);
              w.w = BF16 ? pack_bf16x2(f[6] * m, f[7] * m) : pack_f16x2(f[6] * m, f[7] * m);
              *reinterpret_cast<uint4*>(out + c0 + e) = w;
            }
          }
          // every load of these tiles' dS has completed (their MMAs have): drop the lines
          const uint8_t* base = fp.ds + (int64_t)slot * fp.ds_slot_bytes;
          const int t = threadIdx.x - 64;  // 0 .. 32 EW - 1
          const int lines0 = nkb0 * 128, lines = lines0 + nkb * 128;
          for (int idx = t; idx < lines; idx += 32 * EW) {
            const int j = idx < lines0 ? idx : idx - lines0;
            const int qt = idx < lines0 ? qt0 : qt0 + 1;
            discard_l2_line(base + ((int64_t)(j >> 7) * nqb + qt * 2) * 8192 + (j & 127) * 128);
          }
        }
      }
    }

    // ---------------------------------------------------------------- unit end
    // The workers meet first and a finished dQ unit is counted before the scheduler
    // warp joins: its claim may be waiting for exactly that count (a ticket whose dS
    // slot this unit frees).
    tc_fence_before();
    if (warp != kSchedWarp) {
      named_barrier(1, 32 * (EW + 3));
      if (threadIdx.x == 0) {
        if (*abort) {
          st_relaxed_gpu(&fp.sched[kSchedAbort], 1);
        } else if (*s_kind == 1) {
          __threadfence();  // the discards above are ordered before the slot is handed on
          red_add_release_gpu(&fp.dq_done[unit / (fp.nq / 2)], 1);
        }
      }
    }
    __syncthreads();
    tc_fence_after();
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ===========================================================================
// host
// ===========================================================================

static int env_int(const char* name, int dflt) {
  const char* s = std::getenv(name);
  return (s && *s) ? std::atoi(s) : dflt;
}

static int validate(const char* op, int64_t b, int64_t h, int64_t sq, int64_t sk,
                    int64_t d, int causal, int block_q, int block_k, int dtype) {
  if (b <= 0 || h <= 0 || sq <= 0 || sk <= 0 || d <= 0)
    return fail(FERRITE_BAD_SHAPE, "%s: non-positive shape", op);
  if (d % 128 && d > 128)
    return fail(FERRITE_BAD_SHAPE, "%s: head_dim must be <= 128 or a multiple of it; got %lld", op, (long long)d);
  if (d > kSimtMaxD) return fail(FERRITE_BAD_SHAPE, "%s: head_dim %lld > %d unsupported", op, (long long)d, kSimtMaxD);
  if (causal && sq != sk)
    return fail(FERRITE_BAD_SHAPE, "%s: causal attention needs equal q and k sequence lengths", op);
  if (block_q <= 0 || block_q % 8 || sq % block_q)
    return fail(FERRITE_BAD_SHAPE, "%s: block_q=%d must be a multiple of 8 and divide %lld", op, block_q, (long long)sq);
  if (block_k <= 0 || block_k % 128 || sk % block_k)
    return fail(FERRITE_BAD_SHAPE, "%s: block_k=%d must be a multiple of 128 and divide %lld", op, block_k, (long long)sk);
  if (dtype != FERRITE_F32 && dtype != FERRITE_BF16 && dtype != FERRITE_F16)
    return fail(FERRITE_UNSUPPORTED_DTYPE, "%s: dtype %d", op, dtype);
  if (b * h > 65535) return fail(FERRITE_BAD_SHAPE, "%s: batch*heads > 65535", op);
  if (sq > (1 << 24) || sk > (1 << 24)) return fail(FERRITE_BAD_SHAPE, "%s: sequence too long", op);
  return injected_fault(op);
}

static bool tc_fwd_ok(int64_t d, int64_t sk, int dtype) {
  if (env_int("FERRITE_ATTN_FORCE_SIMT", 0)) return false;
  return dtype != FERRITE_F32 && (d == 64 || d == 128) && sk % TK == 0;
}

// The tensor-core kernels read through TMA and store 16-byte vectors, so every
// operand needs a 16-byte aligned base and strides that are positive multiples
// of 8 (16-bit) elements; an extent-1 dimension's stride is never used.
static bool tc_layout_ok(const void* ptr, const Bhsd& l, int64_t b, int64_t h, int64_t s) {
  if (reinterpret_cast<uintptr_t>(ptr) & 15u) return false;
  auto ok = [](int64_t st, int64_t n) {
    return n == 1 || (st > 0 && st % 8 == 0 && st < (int64_t(1) << 38));
  };
  return ok(l.b, b) && ok(l.h, h) && ok(l.s, s);
}

// 4-D map of a [b, h, s, d] operand: dims (d, s, h, b), box (64, rows, 1, 1),
// 128-byte swizzle.  The smem image of one box is the same [rows][64] K-major
// tile a contiguous 3-D map gives.
static int map_bhsd(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int D,
                    const Bhsd& l, int64_t b, int64_t h, int64_t s, uint32_t rows) {
  auto st = [&](int64_t stride, int64_t n) -> uint64_t {
    return n == 1 ? (uint64_t)D * 2 : (uint64_t)stride * 2;
  };
  const uint64_t dims[4] = {(uint64_t)D, (uint64_t)s, (uint64_t)h, (uint64_t)b};
  const uint64_t strides[3] = {st(l.s, s), st(l.h, h), st(l.b, b)};
  const uint32_t box[4] = {64, rows, 1, 1};
  return make_tmap_4d(m, base, dt, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

template <int D, bool BF16, int NG>
static int launch_fwd_tc_ng(cudaStream_t s, const void* q, const void* k, const void* v,
                         void* o, float* lse, const Bhsd& lq, const Bhsd& lk, const Bhsd& lv,
                         const Bhsd& lo, int64_t b, int64_t h, int64_t sq, int64_t sk,
                         float scale, int causal) {
  using L = FwdSmem<D, NG>;
  const CUtensorMapDataType dt = BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tq, tk, tv;
  int rc = map_bhsd(&tq, q, dt, D, lq, b, h, sq, TQ);
  if (!rc) rc = map_bhsd(&tk, k, dt, D, lk, b, h, sk, TK);
  if (!rc) rc = map_bhsd(&tv, v, dt, D, lv, b, h, sk, TK);
  if (rc) return rc;
  FwdParams p;
  p.sq = (int)sq;
  p.sk = (int)sk;
  p.scale_log2 = scale * kLog2e;
  p.causal = causal;
  p.o = o;
  p.lo = lo;
  p.lse = lse;
  p.nq_blocks = (int)((sq + NG * TQ - 1) / (NG * TQ));
  auto kern = attn_fwd_tc_kernel<D, BF16, NG>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal);
  if (e != cudaSuccess) return fail(FERRITE_LAUNCH_FAILED, "attn_fwd: smem attr: %s", cudaGetErrorString(e));
  dim3 grid(p.nq_blocks, (unsigned)(b * h));
  (void)launch_pdl(kern, dim3(grid), dim3(fwd_threads<NG>()), L::kTotal, s, tq, tk, tv, p);
  return check_launch("attn_fwd_tc");
}

// d = 64 runs one query tile per CTA (two CTAs per SM) unless FERRITE_ATTN_FWD_NG=2;
// d = 128 always pairs two tiles in one CTA (its 1-tile CTA would not fit twice).
template <int D, bool BF16>
static int launch_fwd_tc(cudaStream_t s, const void* q, const void* k, const void* v, void* o,
                         float* lse, const Bhsd& lq, const Bhsd& lk, const Bhsd& lv, const Bhsd& lo,
                         int64_t b, int64_t h, int64_t sq, int64_t sk, float scale, int causal) {
  if constexpr (D == 64) {
    if (env_int("FERRITE_ATTN_FWD_NG", 1) != 2)
      return launch_fwd_tc_ng<D, BF16, 1>(s, q, k, v, o, lse, lq, lk, lv, lo, b, h, sq, sk, scale, causal);
  }
  return launch_fwd_tc_ng<D, BF16, 2>(s, q, k, v, o, lse, lq, lk, lv, lo, b, h, sq, sk, scale, causal);
}

// Operands of one backward call: the four inputs, the outputs and their layouts.
struct BwdArgs {
  const void *q, *k, *v, *dout;
  const float *lse, *delta;
  void *out0, *out1;  // dK, dV (dK/dV kernel) or dQ (dQ kernel)
  Bhsd lq, lk, lv, ldo, l0, l1;
  int64_t bh0 = 0, nbh = -1;  // slice range of the launch (nbh < 0: all)
  void* ds = nullptr;         // dK/dV: optional dS^T output for the slice range
  int64_t ds_ld = 0;
};

// dS^T workspace geometry: [slice][sk][ds_ld] in the input dtype, rows padded to
// whole 64-query tiles.
static int64_t ds_row_elems(int64_t sq) { return (sq + 63) / 64 * 64; }
static int64_t ds_slice_bytes(int64_t sq, int64_t sk) { return ds_row_elems(sq) * sk * 2; }

// dS^T workspace as 64-key x 64-query blocks: block (key block kb, query block
// qb) of slice sl starts at ((sl * sk/64 + kb) * nqb + qb) * 4096 elements, rows
// of 64 queries inside.  4-D tensor map (query, key, query block, slice*key
// block); boxes of `key_rows` keys x `qblocks` query blocks.
static int map_ds_blocks(CUtensorMap* m, const void* ds, CUtensorMapDataType dt, int64_t sq,
                         int64_t sk, int64_t nbh, uint32_t key_rows, uint32_t qblocks) {
  const int64_t nqb = ds_row_elems(sq) / 64;
  const uint64_t dims[4] = {64, 64, (uint64_t)nqb, (uint64_t)(nbh * (sk / 64))};
  const uint64_t strides[3] = {128, 8192, (uint64_t)nqb * 8192};
  const uint32_t box[4] = {64, key_rows, qblocks, 1};
  return make_tmap_4d(m, ds, dt, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

template <int D, bool BF16, bool IS_DKV>
static int launch_bwd_tc(cudaStream_t s, const BwdArgs& a, int64_t b, int64_t h, int64_t sq,
                         int64_t sk, float scale, int causal) {
  using L = BwdSmem<D>;
  const CUtensorMapDataType dt = BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  // stationary pair (128-row boxes) and streaming pair (64-row boxes)
  const int64_t xs = IS_DKV ? sk : sq, ys = IS_DKV ? sq : sk;
  CUtensorMap tx1, tx2, ty1, ty2;
  int rc = map_bhsd(&tx1, IS_DKV ? a.k : a.q, dt, D, IS_DKV ? a.lk : a.lq, b, h, xs, BX);
  if (!rc) rc = map_bhsd(&tx2, IS_DKV ? a.v : a.dout, dt, D, IS_DKV ? a.lv : a.ldo, b, h, xs, BX);
  if (!rc) rc = map_bhsd(&ty1, IS_DKV ? a.q : a.k, dt, D, IS_DKV ? a.lq : a.lk, b, h, ys, BY);
  if (!rc) rc = map_bhsd(&ty2, IS_DKV ? a.dout : a.v, dt, D, IS_DKV ? a.ldo : a.lv, b, h, ys, BY);
  // lse / delta as [bh][sq] f32, 64-query boxes (zero-filled past sq)
  const int64_t bh = b * h;
  CUtensorMap tl, td;
  if (!rc) rc = make_tmap_2d(&tl, a.lse, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)sq, (uint64_t)bh, (uint64_t)sq * 4, BY, 1, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (!rc) rc = make_tmap_2d(&td, a.delta, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)sq, (uint64_t)bh, (uint64_t)sq * 4, BY, 1, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  BwdParams p;
  p.sq = (int)sq;
  p.sk = (int)sk;
  p.scale = scale;
  p.scale_log2 = scale * kLog2e;
  p.causal = causal;
  p.lse = a.lse;
  p.delta = a.delta;
  p.out0 = a.out0;
  p.out1 = a.out1;
  p.l0 = a.l0;
  p.l1 = a.l1;
  p.n_x_tiles = (int)((xs + BX - 1) / BX);
  p.bh0 = (int)a.bh0;
  const int64_t nbh = a.nbh < 0 ? bh - a.bh0 : a.nbh;
  p.ds = IS_DKV ? a.ds : nullptr;
  p.ds_ld = a.ds_ld;
  p.ds_slice = a.ds_ld * sk;
  auto kern = attn_bwd_tc_kernel<D, BF16, IS_DKV>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal);
  if (e != cudaSuccess) return fail(FERRITE_LAUNCH_FAILED, "attn_bwd: smem attr: %s", cudaGetErrorString(e));
  if (nbh <= 0) return FERRITE_OK;
  // dS^T store map over the launch's slices: boxes of 64 queries x 32 keys
  CUtensorMap tds = tl;  // placeholder when no dS is written (never dereferenced)
  if (p.ds) {
    rc = map_ds_blocks(&tds, p.ds, dt, sq, sk, nbh, 32, 1);
    if (rc) return rc;
  }
  dim3 grid(p.n_x_tiles, (unsigned)nbh);
  (void)launch_pdl(kern, dim3(grid), dim3(kBwdThreads), L::kTotal, s, tx1, tx2, ty1, ty2, tl, td, tds, p);
  return check_launch(IS_DKV ? "attn_bwd_dkv_tc" : "attn_bwd_dq_tc");
}

template <int D, bool BF16>
static int launch_dkv_wide(cudaStream_t s, const BwdArgs& a, int64_t b, int64_t h, int64_t sq,
                           int64_t sk, float scale, int causal) {
  using L = WideSmem<D>;
  const CUtensorMapDataType dt = BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tk, tv, tq, tdo;
  int rc = map_bhsd(&tk, a.k, dt, D, a.lk, b, h, sk, BX);
  if (!rc) rc = map_bhsd(&tv, a.v, dt, D, a.lv, b, h, sk, BX);
  if (!rc) rc = map_bhsd(&tq, a.q, dt, D, a.lq, b, h, sq, kWideY);
  if (!rc) rc = map_bhsd(&tdo, a.dout, dt, D, a.ldo, b, h, sq, kWideY);
  // lse / delta as [bh][sq] f32, 128-query boxes (zero-filled past sq)
  const int64_t bh = b * h;
  CUtensorMap tl, td;
  if (!rc) rc = make_tmap_2d(&tl, a.lse, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)sq, (uint64_t)bh, (uint64_t)sq * 4, kWideY, 1, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (!rc) rc = make_tmap_2d(&td, a.delta, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)sq, (uint64_t)bh, (uint64_t)sq * 4, kWideY, 1, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  BwdParams p;
  p.sq = (int)sq;
  p.sk = (int)sk;
  p.scale = scale;
  p.scale_log2 = scale * kLog2e;
  p.causal = causal;
  p.lse = a.lse;
  p.delta = a.delta;
  p.out0 = a.out0;
  p.out1 = a.out1;
  p.l0 = a.l0;
  p.l1 = a.l1;
  p.n_x_tiles = (int)((sk + BX - 1) / BX);
  p.bh0 = (int)a.bh0;
  const int64_t nbh = a.nbh < 0 ? bh - a.bh0 : a.nbh;
  p.ds = a.ds;
  p.ds_ld = a.ds_ld;
  p.ds_slice = a.ds_ld * sk;
  auto kern = attn_dkv_wide_kernel<D, BF16>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal);
  if (e != cudaSuccess) return fail(FERRITE_LAUNCH_FAILED, "attn_bwd_dkv: smem attr: %s", cudaGetErrorString(e));
  if (nbh <= 0) return FERRITE_OK;
  CUtensorMap tds = tl;  // placeholder when no dS is written (never dereferenced)
  if (p.ds) {
    rc = map_ds_blocks(&tds, p.ds, dt, sq, sk, nbh, 32, 1);
    if (rc) return rc;
  }
  dim3 grid(p.n_x_tiles, (unsigned)nbh);
  (void)launch_pdl(kern, dim3(grid), dim3(kWideThreads), L::kTotal, s, tk, tv, tq, tdo, tl, td, tds, p);
  return check_launch("attn_bwd_dkv_wide");
}

template <bool IS_DKV>
static int dispatch_bwd_tc(cudaStream_t s, const BwdArgs& a, int64_t b, int64_t h, int64_t sq,
                           int64_t sk, int64_t d, float scale, int causal, int dtype) {
  const bool bf = dtype == FERRITE_BF16;
  // dK/dV: 128-query tiles (attn_dkv_wide_kernel) unless FERRITE_ATTN_DKV_WIDE=0
  if (IS_DKV && env_int("FERRITE_ATTN_DKV_WIDE", 1) != 0) {
    if (d == 64)
      return bf ? launch_dkv_wide<64, true>(s, a, b, h, sq, sk, scale, causal)
                : launch_dkv_wide<64, false>(s, a, b, h, sq, sk, scale, causal);
    return bf ? launch_dkv_wide<128, true>(s, a, b, h, sq, sk, scale, causal)
              : launch_dkv_wide<128, false>(s, a, b, h, sq, sk, scale, causal);
  }
  if (d == 64)
    return bf ? launch_bwd_tc<64, true, IS_DKV>(s, a, b, h, sq, sk, scale, causal)
              : launch_bwd_tc<64, false, IS_DKV>(s, a, b, h, sq, sk, scale, causal);
  return bf ? launch_bwd_tc<128, true, IS_DKV>(s, a, b, h, sq, sk, scale, causal)
            : launch_bwd_tc<128, false, IS_DKV>(s, a, b, h, sq, sk, scale, causal);
}

template <int D, bool BF16>
static int launch_dq_ds(cudaStream_t s, const BwdArgs& a, int64_t b, int64_t h, int64_t sq,
                        int64_t sk, float scale, int causal) {
  using L = DqSmem<D>;
  const CUtensorMapDataType dt = BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const int64_t nbh = a.nbh < 0 ? b * h - a.bh0 : a.nbh;
  if (nbh <= 0) return FERRITE_OK;
  CUtensorMap tds, tk;
  int rc = map_ds_blocks(&tds, a.ds, dt, sq, sk, nbh, 64, 2);
  if (!rc) rc = map_bhsd(&tk, a.k, dt, D, a.lk, b, h, sk, 64);
  if (rc) return rc;
  DqParams p;
  p.sq = (int)sq;
  p.sk = (int)sk;
  p.causal = causal;
  p.nh = (int)h;
  p.scale = scale;
  p.n_q_tiles = (int)((sq + 127) / 128);
  p.n_slices = (int)nbh;
  p.bh0 = (int)a.bh0;
  p.dq = a.out0;
  p.ldq = a.l0;
  auto kern = attn_dq_ds_kernel<D, BF16>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal);
  if (e != cudaSuccess) return fail(FERRITE_LAUNCH_FAILED, "attn_dq_ds: smem attr: %s", cudaGetErrorString(e));
  const int64_t units = (int64_t)p.n_q_tiles * nbh;
  const int grid = (int)std::min<int64_t>(units, num_sms(current_device()));
  (void)launch_pdl(kern, dim3(grid), dim3(kDqThreads), L::kTotal, s, tds, tk, p);
  return check_launch("attn_dq_ds");
}

static int dispatch_dq_ds(cudaStream_t s, const BwdArgs& a, int64_t b, int64_t h, int64_t sq,
                          int64_t sk, int64_t d, float scale, int causal, int dtype) {
  const bool bf = dtype == FERRITE_BF16;
  if (d == 64)
    return bf ? launch_dq_ds<64, true>(s, a, b, h, sq, sk, scale, causal)
              : launch_dq_ds<64, false>(s, a, b, h, sq, sk, scale, causal);
  return bf ? launch_dq_ds<128, true>(s, a, b, h, sq, sk, scale, causal)
            : launch_dq_ds<128, false>(s, a, b, h, sq, sk, scale, causal);
}

// Fused backward workspace: `slots` dS slots (slice-sized, 8 KiB-aligned blocks)
// followed by the scheduler state (sched ints, ready queue, per-tile producer
// counts, per-slice finished dQ units), 256-byte aligned.
static int64_t fused_sched_bytes(int64_t nslices, int64_t sq) {
  const int64_t ndq = nslices * ((sq + 127) / 128);
  return ((kSchedInts + 2 * ndq + nslices) * 4 + 255) / 256 * 256;
}

// FERRITE_ATTN_BWD_FUSED: 0 never, 1 (default) from 4096 queries on, 2 whenever the
// shape allows.  Below 4096 queries a dK/dV unit is only a few query tiles and the
// unit's fixed costs (barrier set-up, first loads, epilogue) outweigh what the fused
// launch saves: measured on one B200, the two-kernel path took the backward from 1.21
// to 1.00 ms at b64 h16 s1024 d64 (the GPT shape) and from 1.45 to 1.31 ms at d128,
// 3-6% at s2048; the fused kernel was 4% faster at s4096 d64 and level at s8192 d128,
// where it moves less DRAM traffic and takes a rank's slices in one launch.
static bool fused_ok(int64_t sq, int64_t sk, int64_t d, int causal) {
  const int mode = env_int("FERRITE_ATTN_BWD_FUSED", 1);
  if (mode == 0 || (mode == 1 && sq < 4096)) return false;
  if (d != 64 && d != 128) return false;
  if (sq % 256 != 0 || sk % 128 != 0) return false;  // dQ units pair the 128-query tiles
  return !causal || sq == sk;
}

template <int D, bool BF16, int EW>
static int launch_bwd_fused(cudaStream_t s, const BwdArgs& kv, const BwdArgs& qa, int64_t b, int64_t h,
                            int64_t sq, int64_t sk, float scale, int causal, void* workspace,
                            size_t workspace_bytes) {
  using L = FusedSmem<D>;
  const CUtensorMapDataType dt = BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const int64_t bh = b * h;
  const int64_t slot_bytes = ds_slice_bytes(sq, sk);
  const int64_t sched_bytes = fused_sched_bytes(bh, sq);
  const int64_t slots = std::min<int64_t>(bh, ((int64_t)workspace_bytes - sched_bytes) / slot_bytes);
  if (slots < 1) return fail(FERRITE_WORKSPACE_TOO_SMALL, "attn_bwd_fused: workspace below one dS slice + scheduler state");
  CUtensorMap tk, tv, tq, tdo, tl, td, tds_st, tds_ld, tk64;
  int rc = map_bhsd(&tk, kv.k, dt, D, kv.lk, b, h, sk, BX);
  if (!rc) rc = map_bhsd(&tv, kv.v, dt, D, kv.lv, b, h, sk, BX);
  if (!rc) rc = map_bhsd(&tq, kv.q, dt, D, kv.lq, b, h, sq, kWideY);
  if (!rc) rc = map_bhsd(&tdo, kv.dout, dt, D, kv.ldo, b, h, sq, kWideY);
  if (!rc) rc = make_tmap_2d(&tl, kv.lse, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)sq, (uint64_t)bh, (uint64_t)sq * 4, kWideY, 1, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (!rc) rc = make_tmap_2d(&td, kv.delta, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)sq, (uint64_t)bh, (uint64_t)sq * 4, kWideY, 1, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (!rc) rc = map_ds_blocks(&tds_st, workspace, dt, sq, sk, slots, 32, 1);
  if (!rc) rc = map_ds_blocks(&tds_ld, workspace, dt, sq, sk, slots, 64, 2);
  if (!rc) rc = map_bhsd(&tk64, kv.k, dt, D, kv.lk, b, h, sk, 64);
  if (rc) return rc;
  BwdParams p;
  p.sq = (int)sq;
  p.sk = (int)sk;
  p.scale = scale;
  p.scale_log2 = scale * kLog2e;
  p.causal = causal;
  p.lse = kv.lse;
  p.delta = kv.delta;
  p.out0 = kv.out0;
  p.out1 = kv.out1;
  p.l0 = kv.l0;
  p.l1 = kv.l1;
  p.n_x_tiles = (int)(sk / BX);
  p.bh0 = 0;
  p.ds = workspace;
  p.ds_ld = ds_row_elems(sq);
  p.ds_slice = p.ds_ld * sk;
  uint8_t* sched_base = reinterpret_cast<uint8_t*>(workspace) + slots * slot_bytes;
  FusedParams fp;
  fp.nq = (int)(sq / 128);
  fp.nkt = (int)(sk / 128);
  fp.n_slices = (int)bh;
  fp.slots = (int)slots;
  fp.sched = reinterpret_cast<int*>(sched_base);
  fp.ready = fp.sched + kSchedInts;
  fp.row_cnt = fp.ready + bh * fp.nq;
  fp.dq_done = fp.row_cnt + bh * fp.nq;
  fp.ds = reinterpret_cast<uint8_t*>(workspace);
  fp.ds_slot_bytes = slot_bytes;
  fp.dq = qa.out0;
  fp.ldq = qa.l0;
  // scheduler state: counters 0, ready queue -1
  cudaError_t e = cudaMemsetAsync(sched_base, 0, sched_bytes, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(fp.ready, 0xff, (size_t)(bh * (fp.nq / 2)) * 4, s);
  if (e != cudaSuccess) return fail(FERRITE_LAUNCH_FAILED, "attn_bwd_fused: memset: %s", cudaGetErrorString(e));
  auto kern = attn_bwd_fused_kernel<D, BF16, EW>;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal);
  if (e != cudaSuccess) return fail(FERRITE_LAUNCH_FAILED, "attn_bwd_fused: smem attr: %s", cudaGetErrorString(e));
  const int64_t units = bh * (fp.nq / 2 + fp.nkt);
  const int grid = (int)std::min<int64_t>(units, num_sms(current_device()));
  (void)launch_pdl(kern, dim3(grid), dim3(fused_threads<EW>()), L::kTotal, s, tk, tv, tq, tdo, tl, td, tds_st, tds_ld,
                   tk64, p, fp);
  return check_launch("attn_bwd_fused");
}

static int dispatch_bwd_fused(cudaStream_t s, const BwdArgs& kv, const BwdArgs& qa, int64_t b, int64_t h,
                              int64_t sq, int64_t sk, int64_t d, float scale, int causal, int dtype,
                              void* workspace, size_t workspace_bytes) {
  const bool bf = dtype == FERRITE_BF16;
  const bool ew16 = env_int("FERRITE_ATTN_BWD_FUSED_EW", 8) == 16;
#define FUSED(DV, B, E) launch_bwd_fused<DV, B, E>(s, kv, qa, b, h, sq, sk, scale, causal, workspace, workspace_bytes)
  if (d == 64) {
    if (ew16) return bf ? FUSED(64, true, 16) : FUSED(64, false, 16);
    return bf ? FUSED(64, true, 8) : FUSED(64, false, 8);
  }
  if (ew16) return bf ? FUSED(128, true, 16) : FUSED(128, false, 16);
  return bf ? FUSED(128, true, 8) : FUSED(128, false, 8);
#undef FUSED
}

static int strides_ok(const char* op, const ferrite_attn_strides* st) {
  if (!st) return fail(FERRITE_BAD_SHAPE, "%s: null strides", op);
  const int64_t* f = &st->q[0];
  for (int i = 0; i < 24; ++i)
    if (f[i] < 0) return fail(FERRITE_BAD_SHAPE, "%s: negative stride", op);
  return FERRITE_OK;
}

static Bhsd bhsd_of(const int64_t st[3], int64_t h) { return Bhsd{st[0], st[1], st[2], (int)h}; }

static int attn_fwd_impl(cudaStream_t s, const void* q, const void* k, const void* v, void* o,
                         float* lse, const ferrite_attn_strides& st, int64_t b, int64_t h,
                         int64_t sq, int64_t sk, int64_t d, float scale, int causal, int dtype) {
  const Bhsd lq = bhsd_of(st.q, h), lk = bhsd_of(st.k, h), lv = bhsd_of(st.v, h), lo = bhsd_of(st.o, h);
  if (tc_fwd_ok(d, sk, dtype) && tc_layout_ok(q, lq, b, h, sq) && tc_layout_ok(k, lk, b, h, sk) &&
      tc_layout_ok(v, lv, b, h, sk) && tc_layout_ok(o, lo, b, h, sq)) {
    const bool bf = dtype == FERRITE_BF16;
    if (d == 64) return bf ? launch_fwd_tc<64, true>(s, q, k, v, o, lse, lq, lk, lv, lo, b, h, sq, sk, scale, causal)
                           : launch_fwd_tc<64, false>(s, q, k, v, o, lse, lq, lk, lv, lo, b, h, sq, sk, scale, causal);
    return bf ? launch_fwd_tc<128, true>(s, q, k, v, o, lse, lq, lk, lv, lo, b, h, sq, sk, scale, causal)
              : launch_fwd_tc<128, false>(s, q, k, v, o, lse, lq, lk, lv, lo, b, h, sq, sk, scale, causal);
  }
  dim3 grid((unsigned)((sq + kSimtWarps - 1) / kSimtWarps), (unsigned)(b * h));
#define FWD(T)                                                                                  \
  (void)launch_pdl(simt_fwd_kernel<T>, dim3(grid), dim3(kSimtWarps * 32), 0, s, (const T*)q, (const T*)k, (const T*)v,    \
                                                       (T*)o, lse, lq, lk, lv, lo, (int)sq,     \
                                                       (int)sk, (int)d, scale, causal)
  if (dtype == FERRITE_F32) FWD(float);
  else if (dtype == FERRITE_BF16) FWD(__nv_bfloat16);
  else FWD(__half);
#undef FWD
  return check_launch("attn_fwd_simt");
}

template <typename T>
static bool prep_vec_ok(const void* p, const Bhsd& l, int64_t b, int64_t h) {
  constexpr int kElems = 16 / sizeof(T);
  auto ok = [](int64_t st, int64_t n) { return n == 1 || st % kElems == 0; };
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0 && l.s % kElems == 0 && ok(l.b, b) && ok(l.h, h);
}

template <typename T>
static int launch_prep(cudaStream_t s, const void* dout, const void* out, float* delta,
                       const Bhsd& ld, const Bhsd& lo, int64_t b, int64_t h, int64_t s_, int64_t d) {
  constexpr int kElems = 16 / sizeof(T);
  const int64_t vpr = d / kElems;
  const bool vec = d % kElems == 0 && vpr <= 32 && (vpr & (vpr - 1)) == 0 && b * h <= 65535 &&
                   prep_vec_ok<T>(dout, ld, b, h) && prep_vec_ok<T>(out, lo, b, h);
  if (vec) {
    const int rpc = prep_rows_per_cta((int)vpr);
    dim3 grid((unsigned)((s_ + rpc - 1) / rpc), (unsigned)(b * h));
    const T* a = (const T*)dout;
    const T* o = (const T*)out;
    switch (vpr) {
      case 1: (void)launch_pdl(bwd_prep_vec_kernel<T, 1>, dim3(grid), dim3(256), 0, s, a, o, delta, ld, lo, (int)s_); break;
      case 2: (void)launch_pdl(bwd_prep_vec_kernel<T, 2>, dim3(grid), dim3(256), 0, s, a, o, delta, ld, lo, (int)s_); break;
      case 4: (void)launch_pdl(bwd_prep_vec_kernel<T, 4>, dim3(grid), dim3(256), 0, s, a, o, delta, ld, lo, (int)s_); break;
      case 8: (void)launch_pdl(bwd_prep_vec_kernel<T, 8>, dim3(grid), dim3(256), 0, s, a, o, delta, ld, lo, (int)s_); break;
      case 16: (void)launch_pdl(bwd_prep_vec_kernel<T, 16>, dim3(grid), dim3(256), 0, s, a, o, delta, ld, lo, (int)s_); break;
      default: (void)launch_pdl(bwd_prep_vec_kernel<T, 32>, dim3(grid), dim3(256), 0, s, a, o, delta, ld, lo, (int)s_); break;
    }
    return check_launch("attn_bwd_prep");
  }
  const int64_t rows = b * h * s_;
  (void)launch_pdl(bwd_prep_kernel<T>, dim3((unsigned)((rows + 7) / 8)), dim3(256), 0, s, (const T*)dout, (const T*)out, delta, ld,
                                                                 lo, rows, (int)s_, (int)d);
  return check_launch("attn_bwd_prep");
}

static int attn_bwd_prep_impl(cudaStream_t s, const void* dout, const void* out, float* delta,
                              const ferrite_attn_strides& st, int64_t b, int64_t h, int64_t s_,
                              int64_t d, int dtype) {
  const Bhsd ld = bhsd_of(st.dout, h), lo = bhsd_of(st.o, h);
  if (dtype == FERRITE_F32) return launch_prep<float>(s, dout, out, delta, ld, lo, b, h, s_, d);
  if (dtype == FERRITE_BF16) return launch_prep<__nv_bfloat16>(s, dout, out, delta, ld, lo, b, h, s_, d);
  if (dtype == FERRITE_F16) return launch_prep<__half>(s, dout, out, delta, ld, lo, b, h, s_, d);
  return fail(FERRITE_UNSUPPORTED_DTYPE, "attn_bwd_prep: dtype %d", dtype);
}

static bool tc_bwd_ok(const BwdArgs& a, int64_t b, int64_t h, int64_t sq, int64_t sk, int64_t d,
                      int dtype, bool is_dkv) {
  if (!tc_fwd_ok(d, sk, dtype) || env_int("FERRITE_ATTN_BWD_FORCE_SIMT", 0)) return false;
  bool ok = tc_layout_ok(a.q, a.lq, b, h, sq) && tc_layout_ok(a.k, a.lk, b, h, sk) &&
            tc_layout_ok(a.v, a.lv, b, h, sk) && tc_layout_ok(a.dout, a.ldo, b, h, sq);
  if (is_dkv) return ok && tc_layout_ok(a.out0, a.l0, b, h, sk) && tc_layout_ok(a.out1, a.l1, b, h, sk);
  return ok && tc_layout_ok(a.out0, a.l0, b, h, sq);
}

static int attn_bwd_dkv_impl(cudaStream_t s, const BwdArgs& a, int64_t b, int64_t h, int64_t sq,
                             int64_t sk, int64_t d, float scale, int causal, int dtype) {
  if (tc_bwd_ok(a, b, h, sq, sk, d, dtype, true))
    return dispatch_bwd_tc<true>(s, a, b, h, sq, sk, d, scale, causal, dtype);
  dim3 grid((unsigned)((sk + kSimtWarps - 1) / kSimtWarps), (unsigned)(b * h));
#define DKV(T)                                                                                  \
  (void)launch_pdl(simt_bwd_dkv_kernel<T>, dim3(grid), dim3(kSimtWarps * 32), 0, s,                                       \
      (const T*)a.q, (const T*)a.k, (const T*)a.v, (const T*)a.dout, a.lse, a.delta,            \
      (T*)a.out0, (T*)a.out1, a.lq, a.lk, a.lv, a.ldo, a.l0, a.l1, (int)sq, (int)sk, (int)d,    \
      scale, causal)
  if (dtype == FERRITE_F32) DKV(float);
  else if (dtype == FERRITE_BF16) DKV(__nv_bfloat16);
  else DKV(__half);
#undef DKV
  return check_launch("attn_bwd_dkv_simt");
}

static int attn_bwd_dq_impl(cudaStream_t s, const BwdArgs& a, int64_t b, int64_t h, int64_t sq,
                            int64_t sk, int64_t d, float scale, int causal, int dtype) {
  if (tc_bwd_ok(a, b, h, sq, sk, d, dtype, false))
    return dispatch_bwd_tc<false>(s, a, b, h, sq, sk, d, scale, causal, dtype);
  dim3 grid((unsigned)((sq + kSimtWarps - 1) / kSimtWarps), (unsigned)(b * h));
#define DQ(T)                                                                                    \
  (void)launch_pdl(simt_bwd_dq_kernel<T>, dim3(grid), dim3(kSimtWarps * 32), 0, s,                                         \
      (const T*)a.q, (const T*)a.k, (const T*)a.v, (const T*)a.dout, a.lse, a.delta, (T*)a.out0, \
      a.lq, a.lk, a.lv, a.ldo, a.l0, (int)sq, (int)sk, (int)d, scale, causal)
  if (dtype == FERRITE_F32) DQ(float);
  else if (dtype == FERRITE_BF16) DQ(__nv_bfloat16);
  else DQ(__half);
#undef DQ
  return check_launch("attn_bwd_dq_simt");
}

static ferrite_attn_strides contiguous_strides(int64_t h, int64_t sq, int64_t sk, int64_t d) {
  ferrite_attn_strides st;
  auto set = [](int64_t* f, int64_t h_, int64_t s_, int64_t d_) {
    f[0] = h_ * s_ * d_;
    f[1] = s_ * d_;
    f[2] = d_;
  };
  set(st.q, h, sq, d);
  set(st.o, h, sq, d);
  set(st.dout, h, sq, d);
  set(st.dq, h, sq, d);
  set(st.k, h, sk, d);
  set(st.v, h, sk, d);
  set(st.dk, h, sk, d);
  set(st.dv, h, sk, d);
  return st;
}

static BwdArgs bwd_args(const void* q, const void* k, const void* v, const void* dout,
                        const float* lse, const float* delta, void* out0, void* out1,
                        const ferrite_attn_strides& st, int64_t h, bool is_dkv) {
  BwdArgs a;
  a.q = q;
  a.k = k;
  a.v = v;
  a.dout = dout;
  a.lse = lse;
  a.delta = delta;
  a.out0 = out0;
  a.out1 = out1;
  a.lq = bhsd_of(st.q, h);
  a.lk = bhsd_of(st.k, h);
  a.lv = bhsd_of(st.v, h);
  a.ldo = bhsd_of(st.dout, h);
  a.l0 = bhsd_of(is_dkv ? st.dk : st.dq, h);
  a.l1 = bhsd_of(st.dv, h);
  return a;
}

}  // namespace attn
}  // namespace ferrite

using namespace ferrite;
using namespace ferrite::attn;

extern "C" {

int ferrite_attn_fwd_strided(void* stream, const void* q, const void* k, const void* v, void* o,
                             float* lse, const ferrite_attn_strides* st, int64_t b, int64_t h,
                             int64_t sq, int64_t sk, int64_t d, float scale, int causal,
                             int block_q, int block_k, int dtype) {
  if (int rc = validate("attn_fwd", b, h, sq, sk, d, causal, block_q, block_k, dtype)) return rc;
  if (!q || !k || !v || !o || !lse) return fail(FERRITE_BAD_SHAPE, "attn_fwd: null pointer");
  if (int rc = strides_ok("attn_fwd", st)) return rc;
  return attn_fwd_impl((cudaStream_t)stream, q, k, v, o, lse, *st, b, h, sq, sk, d, scale, causal, dtype);
}

int ferrite_attn_fwd(void* stream, const void* q, const void* k, const void* v, void* o,
                     float* lse, int64_t b, int64_t h, int64_t sq, int64_t sk, int64_t d,
                     float scale, int causal, int block_q, int block_k, int dtype) {
  const ferrite_attn_strides st = contiguous_strides(h, sq, sk, d);
  return ferrite_attn_fwd_strided(stream, q, k, v, o, lse, &st, b, h, sq, sk, d, scale, causal,
                                  block_q, block_k, dtype);
}

int ferrite_attn_bwd_prep_strided(void* stream, const void* dout, const void* out, float* delta,
                                  const ferrite_attn_strides* st, int64_t b, int64_t h, int64_t s_,
                                  int64_t d, int dtype) {
  if (int rc = injected_fault("attn_bwd_prep")) return rc;
  if (b <= 0 || h <= 0 || s_ <= 0 || d <= 0) return fail(FERRITE_BAD_SHAPE, "attn_bwd_prep: shape");
  if (!dout || !out || !delta) return fail(FERRITE_BAD_SHAPE, "attn_bwd_prep: null pointer");
  if (int rc = strides_ok("attn_bwd_prep", st)) return rc;
  return attn_bwd_prep_impl((cudaStream_t)stream, dout, out, delta, *st, b, h, s_, d, dtype);
}

int ferrite_attn_bwd_prep(void* stream, const void* dout, const void* out, float* delta,
                          int64_t b, int64_t h, int64_t s_, int64_t d, int dtype) {
  const ferrite_attn_strides st = contiguous_strides(h, s_, s_, d);
  return ferrite_attn_bwd_prep_strided(stream, dout, out, delta, &st, b, h, s_, d, dtype);
}

int ferrite_attn_bwd_dkv_strided(void* stream, const void* q, const void* k, const void* v,
                                 const void* dout, const float* lse, const float* delta, void* dk,
                                 void* dv, const ferrite_attn_strides* st, int64_t b, int64_t h,
                                 int64_t sq, int64_t sk, int64_t d, float scale, int causal,
                                 int block_q, int block_k, int dtype) {
  if (int rc = validate("attn_bwd_dkv", b, h, sq, sk, d, causal, block_q, block_k, dtype)) return rc;
  if (!q || !k || !v || !dout || !lse || !delta || !dk || !dv)
    return fail(FERRITE_BAD_SHAPE, "attn_bwd_dkv: null pointer");
  if (int rc = strides_ok("attn_bwd_dkv", st)) return rc;
  const BwdArgs a = bwd_args(q, k, v, dout, lse, delta, dk, dv, *st, h, true);
  return attn_bwd_dkv_impl((cudaStream_t)stream, a, b, h, sq, sk, d, scale, causal, dtype);
}

int ferrite_attn_bwd_dkv(void* stream, const void* q, const void* k, const void* v,
                         const void* dout, const float* lse, const float* delta, void* dk,
                         void* dv, int64_t b, int64_t h, int64_t sq, int64_t sk, int64_t d,
                         float scale, int causal, int block_q, int block_k, int dtype) {
  const ferrite_attn_strides st = contiguous_strides(h, sq, sk, d);
  return ferrite_attn_bwd_dkv_strided(stream, q, k, v, dout, lse, delta, dk, dv, &st, b, h, sq, sk,
                                      d, scale, causal, block_q, block_k, dtype);
}

int ferrite_attn_bwd_dq_strided(void* stream, const void* q, const void* k, const void* v,
                                const void* dout, const float* lse, const float* delta, void* dq,
                                const ferrite_attn_strides* st, int64_t b, int64_t h, int64_t sq,
                                int64_t sk, int64_t d, float scale, int causal, int block_q,
                                int block_k, int dtype) {
  if (int rc = validate("attn_bwd_dq", b, h, sq, sk, d, causal, block_q, block_k, dtype)) return rc;
  if (!q || !k || !v || !dout || !lse || !delta || !dq)
    return fail(FERRITE_BAD_SHAPE, "attn_bwd_dq: null pointer");
  if (int rc = strides_ok("attn_bwd_dq", st)) return rc;
  const BwdArgs a = bwd_args(q, k, v, dout, lse, delta, dq, nullptr, *st, h, false);
  return attn_bwd_dq_impl((cudaStream_t)stream, a, b, h, sq, sk, d, scale, causal, dtype);
}

int ferrite_attn_bwd_dq(void* stream, const void* q, const void* k, const void* v,
                        const void* dout, const float* lse, const float* delta, void* dq,
                        int64_t b, int64_t h, int64_t sq, int64_t sk, int64_t d, float scale,
                        int causal, int block_q, int block_k, int dtype) {
  const ferrite_attn_strides st = contiguous_strides(h, sq, sk, d);
  return ferrite_attn_bwd_dq_strided(stream, q, k, v, dout, lse, delta, dq, &st, b, h, sq, sk, d,
                                     scale, causal, block_q, block_k, dtype);
}

int ferrite_attn_bwd_dkv_ds(void* stream, const void* q, const void* k, const void* v,
                            const void* dout, const float* lse, const float* delta, void* dk,
                            void* dv, void* ds, const ferrite_attn_strides* st, int64_t bh_begin,
                            int64_t bh_count, int64_t b, int64_t h, int64_t sq, int64_t sk,
                            int64_t d, float scale, int causal, int block_q, int block_k,
                            int dtype) {
  if (int rc = validate("attn_bwd_dkv_ds", b, h, sq, sk, d, causal, block_q, block_k, dtype)) return rc;
  if (!q || !k || !v || !dout || !lse || !delta || !dk || !dv || !ds)
    return fail(FERRITE_BAD_SHAPE, "attn_bwd_dkv_ds: null pointer");
  if (int rc = strides_ok("attn_bwd_dkv_ds", st)) return rc;
  if (bh_begin < 0 || bh_count < 0 || bh_begin + bh_count > b * h)
    return fail(FERRITE_BAD_SHAPE, "attn_bwd_dkv_ds: slice range [%lld, +%lld) outside b*h",
                (long long)bh_begin, (long long)bh_count);
  BwdArgs a = bwd_args(q, k, v, dout, lse, delta, dk, dv, *st, h, true);
  if (!tc_bwd_ok(a, b, h, sq, sk, d, dtype, true) || (reinterpret_cast<uintptr_t>(ds) & 255u))
    return fail(FERRITE_UNSUPPORTED_DTYPE,
                "attn_bwd_dkv_ds: needs the tensor-core path (bf16/f16, d 64/128, sk %% 128 == 0, "
                "16-byte aligned operands, 256-byte aligned dS)");
  a.bh0 = bh_begin;
  a.nbh = bh_count;
  a.ds = ds;
  a.ds_ld = ds_row_elems(sq);
  return dispatch_bwd_tc<true>((cudaStream_t)stream, a, b, h, sq, sk, d, scale, causal, dtype);
}

int ferrite_attn_bwd_dq_ds(void* stream, const void* ds, const void* k, void* dq,
                           const ferrite_attn_strides* st, int64_t bh_begin, int64_t bh_count,
                           int64_t b, int64_t h, int64_t sq, int64_t sk, int64_t d, float scale,
                           int causal, int block_q, int block_k, int dtype) {
  if (int rc = validate("attn_bwd_dq_ds", b, h, sq, sk, d, causal, block_q, block_k, dtype)) return rc;
  if (!ds || !k || !dq) return fail(FERRITE_BAD_SHAPE, "attn_bwd_dq_ds: null pointer");
  if (int rc = strides_ok("attn_bwd_dq_ds", st)) return rc;
  if (bh_begin < 0 || bh_count < 0 || bh_begin + bh_count > b * h)
    return fail(FERRITE_BAD_SHAPE, "attn_bwd_dq_ds: slice range [%lld, +%lld) outside b*h",
                (long long)bh_begin, (long long)bh_count);
  BwdArgs a = bwd_args(nullptr, k, nullptr, nullptr, nullptr, nullptr, dq, nullptr, *st, h, false);
  if (!tc_fwd_ok(d, sk, dtype) || !tc_layout_ok(k, a.lk, b, h, sk) ||
      !tc_layout_ok(dq, a.l0, b, h, sq) || (reinterpret_cast<uintptr_t>(ds) & 255u))
    return fail(FERRITE_UNSUPPORTED_DTYPE,
                "attn_bwd_dq_ds: needs the tensor-core path (bf16/f16, d 64/128, sk %% 128 == 0, "
                "16-byte aligned operands, 256-byte aligned dS)");
  a.bh0 = bh_begin;
  a.nbh = bh_count;
  a.ds = const_cast<void*>(ds);
  a.ds_ld = ds_row_elems(sq);
  return dispatch_dq_ds((cudaStream_t)stream, a, b, h, sq, sk, d, scale, causal, dtype);
}

size_t ferrite_attn_bwd_ds_workspace_size(int64_t b, int64_t h, int64_t sq, int64_t sk,
                                          int64_t d, int dtype) {
  if (b <= 0 || h <= 0 || sq <= 0 || sk <= 0 || !tc_fwd_ok(d, sk, dtype)) return 0;
  return (size_t)(b * h) * (size_t)ds_slice_bytes(sq, sk) + (size_t)fused_sched_bytes(b * h, sq);
}

int ferrite_attn_bwd_ds(void* stream, const void* q, const void* k, const void* v,
                        const void* dout, const float* lse, const float* delta, void* dq,
                        void* dk, void* dv, const ferrite_attn_strides* st, void* workspace,
                        size_t workspace_bytes, int64_t b, int64_t h, int64_t sq, int64_t sk,
                        int64_t d, float scale, int causal, int block_q, int block_k,
                        int dtype) {
  if (int rc = validate("attn_bwd_ds", b, h, sq, sk, d, causal, block_q, block_k, dtype)) return rc;
  if (!q || !k || !v || !dout || !lse || !delta || !dq || !dk || !dv)
    return fail(FERRITE_BAD_SHAPE, "attn_bwd_ds: null pointer");
  if (int rc = strides_ok("attn_bwd_ds", st)) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  BwdArgs kv = bwd_args(q, k, v, dout, lse, delta, dk, dv, *st, h, true);
  BwdArgs qa = bwd_args(q, k, v, dout, lse, delta, dq, nullptr, *st, h, false);
  const int64_t slice = ds_slice_bytes(sq, sk);
  const int64_t per = workspace ? (int64_t)(workspace_bytes / (size_t)slice) : 0;
  const bool use_ds = per >= 1 && (reinterpret_cast<uintptr_t>(workspace) & 255u) == 0 &&
                      env_int("FERRITE_ATTN_BWD_DS", 1) != 0 &&
                      tc_bwd_ok(kv, b, h, sq, sk, d, dtype, true) &&
                      tc_bwd_ok(qa, b, h, sq, sk, d, dtype, false);
  if (!use_ds) {  // recompute path: dK/dV and dQ kernels over all slices
    if (int rc = attn_bwd_dkv_impl(s, kv, b, h, sq, sk, d, scale, causal, dtype)) return rc;
    return attn_bwd_dq_impl(s, qa, b, h, sq, sk, d, scale, causal, dtype);
  }
  const int64_t bh = b * h;
  if (fused_ok(sq, sk, d, causal) &&
      (int64_t)workspace_bytes >= ds_slice_bytes(sq, sk) + fused_sched_bytes(bh, sq))
    return dispatch_bwd_fused(s, kv, qa, b, h, sq, sk, d, scale, causal, dtype, workspace, workspace_bytes);
  // two launches per chunk of slices; chunks of equal size (32 slices in a budget of 31
  // run as 16 + 16, not 31 + 1, whose second launch would leave most SMs idle)
  const int64_t nchunks = (bh + per - 1) / per;
  const int64_t chunk = (bh + nchunks - 1) / nchunks;
  for (int64_t bh0 = 0; bh0 < bh; bh0 += chunk) {
    const int64_t n = std::min<int64_t>(chunk, bh - bh0);
    kv.bh0 = qa.bh0 = bh0;
    kv.nbh = qa.nbh = n;
    kv.ds = qa.ds = workspace;
    kv.ds_ld = qa.ds_ld = ds_row_elems(sq);
    if (int rc = dispatch_bwd_tc<true>(s, kv, b, h, sq, sk, d, scale, causal, dtype)) return rc;
    if (int rc = dispatch_dq_ds(s, qa, b, h, sq, sk, d, scale, causal, dtype)) return rc;
  }
  return FERRITE_OK;
}

}  // extern "C"
