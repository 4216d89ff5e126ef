// Matmul with an f32 accumulator for sm_100a.
//
// bf16/f16 operands: persistent, warp-specialised tcgen05 kernels.  Plans with
// 256-wide tiles and M >= 256 run on CTA pairs (gemm_tc2_kernel, below: one
// 256 x 256 tile per cluster of two CTAs with cta_group::2 MMAs); the rest on
// one CTA per 128-row tile (gemm_tc_kernel), described here:
//   * warp 0 (one elected lane) issues TMA loads of A and B tiles into a ring of
//     STAGES shared-memory slots (128-byte swizzle, no padding copies: ragged
//     edges are zero-filled by TMA);
//   * warp 1 owns the TMEM allocation and (one lane) issues tcgen05.mma
//     (M=128, N=BN, K=16, kind::f16) into an f32 accumulator in TMEM; every slot
//     is released with tcgen05.commit -> mbarrier, every finished tile with a
//     commit to the accumulator's "full" barrier;
//   * warps 2-9 are the epilogue, two per TMEM lane quarter (each half of the
//     tile's columns): tcgen05.ld the accumulator (two TMEM buffers, so the
//     epilogue of tile i overlaps the main loop of tile i+1), convert (and apply
//     the fused activation epilogues), and store: 16-bit outputs go through
//     per-warp 32 x 32 shared-memory staging slots and TMA stores (one store
//     instruction per chunk instead of 32 scattered row writes per warp store;
//     the unit clips M / N edges), f32 outputs with masked vector stores.
//   Operands may be K-major or MN-major in global memory (the transpose flags
//   of the C ABI); the MN-major case uses MN-major shared-memory layouts and the
//   instruction descriptor's transpose bits instead of materialised transposes.
//   Split-K: when the output has too few tiles to fill the SMs (the weight
//   gradients X^T G of a transformer: small M x N, K = tokens), each tile's K
//   range is cut into `splits` slices that run as independent work units and
//   write f32 partial tiles to a caller-provided workspace; a second kernel sums
//   the slices in slice order (deterministic, no atomics) and rounds once.
//
// f32 operands (the reference's Precision.HIGHEST contract, _compat.py:17-26)
// and shapes TMA cannot describe (row strides not a multiple of 16 bytes, tiny
// dimensions) run a register-tiled CUDA-core kernel that accumulates in f32 with
// FFMA: exact f32 products, no reduced-precision passes.
//
// Reference: src/ferrite/kernels/matmul.py of anxnd2211/ferrite-tpu
// (_matmul_kernel :27-38, _matmul_impl :52-86, VJP :99-104).
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "common.cuh"

namespace ferrite {
FERRITE_DEFINE_STATUS_READER(status_gemm)

namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 x 16-bit = 128 bytes: one swizzle row
constexpr int kEpiWarps = 8;  // two warps per TMEM lane quarter, each half of the columns
constexpr int kThreads = 64 + 32 * kEpiWarps;

template <int BN>
struct Smem {
  static constexpr int kStages = BN == 256 ? 4 : 6;
  static constexpr int kABytes = BM * BK * 2;  // 16 KiB
  static constexpr int kBBytes = BN * BK * 2;  // 16 or 32 KiB
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTileBytes = kStages * kStageBytes;
  // 16-bit outputs leave through TMA stores: per epilogue warp two 32 x 32 staging
  // slots (2 KiB each, 64-byte swizzle), alternating so the store of one chunk
  // overlaps the conversion of the next.
  static constexpr int kSlotBytes = 32 * 32 * 2;
  static constexpr int kStgOff = kTileBytes;
  static constexpr int kStgBytes = kEpiWarps * 2 * kSlotBytes;
  // barriers: full[S], empty[S], acc_full[2], acc_empty[2]; then tmem base, abort
  static constexpr int kBarOff = kStgOff + kStgBytes;
  static constexpr int kBarBytes = (2 * kStages + 4) * 8 + 16;
  static constexpr int kTotal = 1024 /*alignment slack*/ + kBarOff + kBarBytes;
};

struct Params {
  int m, n, k;
  int64_t ldc;
  void* c;
  int tiles_m, tiles_n, k_blocks;
  int group_m;  // raster: groups of group_m M-tiles sweep all N-tiles
  int splits;        // K slices per tile (1: no split)
  int kb_per_split;  // k blocks per slice
  float* ws;         // splits > 1: f32 partials [splits][m][n]
  void* aux;         // epilogue operand (GELU: the activation output / the pre-activation input)
  int64_t ld_aux;
  int tma_store;     // 16-bit C (and aux output) written through tensor maps
};

template <typename TC>
__device__ __forceinline__ void store_row32(TC* __restrict__ c, int64_t ldc, int row,
                                            int col0, int m, int n, const uint32_t (&r)[32],
                                            bool vec_ok) {
  if (row >= m) return;
  TC* dst = c + (int64_t)row * ldc + col0;
  if (vec_ok && col0 + 32 <= n) {
    if constexpr (sizeof(TC) == 2) {
#pragma unroll
      for (int j = 0; j < 32; j += 8) {
        uint4 v;
        if constexpr (std::is_same<TC, __nv_bfloat16>::value) {
          v.x = pack_bf16x2(__uint_as_float(r[j]), __uint_as_float(r[j + 1]));
          v.y = pack_bf16x2(__uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
          v.z = pack_bf16x2(__uint_as_float(r[j + 4]), __uint_as_float(r[j + 5]));
          v.w = pack_bf16x2(__uint_as_float(r[j + 6]), __uint_as_float(r[j + 7]));
        } else {
          v.x = pack_f16x2(__uint_as_float(r[j]), __uint_as_float(r[j + 1]));
          v.y = pack_f16x2(__uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
          v.z = pack_f16x2(__uint_as_float(r[j + 4]), __uint_as_float(r[j + 5]));
          v.w = pack_f16x2(__uint_as_float(r[j + 6]), __uint_as_float(r[j + 7]));
        }
        *reinterpret_cast<uint4*>(dst + j) = v;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        *reinterpret_cast<uint4*>(dst + j) = make_uint4(r[j], r[j + 1], r[j + 2], r[j + 3]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (col0 + j < n) dst[j] = DT<TC>::from_f(__uint_as_float(r[j]));
  }
}

// Epilogues (bf16/f16 outputs, unsplit K):
//   kEpiNone     C = acc
//   kEpiGelu     C = u = round(acc); aux = round(gelu_tanh(u))  (the MLP up-projection
//                and its activation, gpt.py:141, in one pass)
//   kEpiGeluBwd  C = round(round(acc) * gelu_tanh'(aux))        (the activation's
//                backward folded into the dA = dP W2^T product; aux = u)
constexpr int kEpiNone = 0, kEpiGelu = 1, kEpiGeluBwd = 2;

// tanh-approximated GELU and its derivative in f32 (the formula of
// jax.nn.gelu(approximate=True) / torch gelu(approximate="tanh")), evaluated via
// the identity 1 + tanh(y) = 2 sigmoid(2y): with y = sqrt(2/pi) (x + 0.044715 x^3)
// and s = 1 / (1 + e^(-2y)),
//   gelu(x)  = x s
//   gelu'(x) = s + 2 x s (1 - s) sqrt(2/pi) (1 + 3 * 0.044715 x^2)
// (1 - tanh^2 = 4 s (1 - s)).  Two MUFU operations per element and no
// cancellation for large |x|; agrees with the tanh form to ~1e-6 relative.
__device__ __forceinline__ float gelu_sigmoid_arg(float x) {  // s
  const float kBeta = 0.7978845608028654f;  // sqrt(2 / pi)
  const float y = kBeta * fmaf(0.044715f * x, x * x, x);
  float e;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(-2.8853900817779268f * y));  // e^(-2y)
  return __fdividef(1.0f, 1.0f + e);
}
__device__ __forceinline__ float gelu_tanh_f(float x) { return x * gelu_sigmoid_arg(x); }
__device__ __forceinline__ float gelu_tanh_grad_f(float x) {
  const float kBeta = 0.7978845608028654f;
  const float s = gelu_sigmoid_arg(x);
  return fmaf(2.0f * x * s * (1.0f - s), kBeta * fmaf(3.0f * 0.044715f * x, x, 1.0f), s);
}

// Rows of 32 accumulator columns through an epilogue: r holds f32 bits on entry.
template <typename TC, int EPI>
__device__ __forceinline__ void epilogue_row32(const Params& p, TC* c, int row, int col0,
                                               uint32_t (&r)[32], bool vec_ok) {
  if constexpr (EPI == kEpiNone) {
    store_row32<TC>(c, p.ldc, row, col0, p.m, p.n, r, vec_ok);
  } else {
    if (row >= p.m) return;
    TC* aux = reinterpret_cast<TC*>(p.aux) + (int64_t)row * p.ld_aux + col0;
    const bool aux_vec = ((reinterpret_cast<uintptr_t>(p.aux) & 15u) == 0) &&
                         ((p.ld_aux * (int64_t)sizeof(TC)) % 16 == 0);
    if constexpr (EPI == kEpiGelu) {
      uint32_t a[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float u = DT<TC>::to_f(DT<TC>::from_f(__uint_as_float(r[j])));
        a[j] = __float_as_uint(gelu_tanh_f(u));
      }
      store_row32<TC>(c, p.ldc, row, col0, p.m, p.n, r, vec_ok);
      store_row32<TC>(aux, 0, 0, 0, 1, p.n - col0, a, aux_vec);
    } else {
      float u[32];
      if (aux_vec && col0 + 32 <= p.n) {
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          const uint4 v = *reinterpret_cast<const uint4*>(aux + j);
          const TC* e = reinterpret_cast<const TC*>(&v);
#pragma unroll
          for (int t = 0; t < 8; ++t) u[j + t] = DT<TC>::to_f(e[t]);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) u[j] = col0 + j < p.n ? DT<TC>::to_f(aux[j]) : 0.f;
      }
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float da = DT<TC>::to_f(DT<TC>::from_f(__uint_as_float(r[j])));
        r[j] = __float_as_uint(da * gelu_tanh_grad_f(u[j]));
      }
      store_row32<TC>(c, p.ldc, row, col0, p.m, p.n, r, vec_ok);
    }
  }
}

// Stage a warp's 32 rows x 32 columns (f32 bits in r, one row per lane) into
// staging slot (count & 1) as 16-bit values with the 64-byte swizzle (16-byte
// chunk c of row l at c ^ ((l >> 1) & 3): conflict-free), then lane 0 issues the
// TMA store of the 32 x 32 box at (x, y).  Before a slot is rewritten, the
// store issued from it two chunks earlier must have finished reading it.
template <typename TC>
__device__ __forceinline__ void stage_store_32x32(uint8_t* stg_base, int ew, int count, int lane,
                                                  const uint32_t (&r)[32], const CUtensorMap* map,
                                                  int x, int y) {
  uint8_t* slot = stg_base + (ew * 2 + (count & 1)) * (32 * 32 * 2);
  if (lane == 0) bulk_wait_group_read1();
  __syncwarp();
  uint8_t* row = slot + lane * 64;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint4 v;
    const int j = c * 8;
    if constexpr (std::is_same<TC, __nv_bfloat16>::value) {
      v.x = pack_bf16x2(__uint_as_float(r[j]), __uint_as_float(r[j + 1]));
      v.y = pack_bf16x2(__uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
      v.z = pack_bf16x2(__uint_as_float(r[j + 4]), __uint_as_float(r[j + 5]));
      v.w = pack_bf16x2(__uint_as_float(r[j + 6]), __uint_as_float(r[j + 7]));
    } else {
      v.x = pack_f16x2(__uint_as_float(r[j]), __uint_as_float(r[j + 1]));
      v.y = pack_f16x2(__uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
      v.z = pack_f16x2(__uint_as_float(r[j + 4]), __uint_as_float(r[j + 5]));
      v.w = pack_f16x2(__uint_as_float(r[j + 6]), __uint_as_float(r[j + 7]));
    }
    *reinterpret_cast<uint4*>(row + ((c ^ ((lane >> 1) & 3)) << 4)) = v;
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(map, slot, x, y);
    bulk_commit_group();
  }
}

// GELU backward values for a 32-column chunk of one row: r (f32 bits of dA, in)
// becomes round(dA) * gelu'(u) with u read from aux.
template <typename TC>
__device__ __forceinline__ void epilogue_gelu_bwd_vals(const Params& p, int row, int col0,
                                                       uint32_t (&r)[32]) {
  float u[32];
  const TC* aux = reinterpret_cast<const TC*>(p.aux) + (int64_t)row * p.ld_aux + col0;
  const bool aux_vec = ((reinterpret_cast<uintptr_t>(p.aux) & 15u) == 0) &&
                       ((p.ld_aux * (int64_t)sizeof(TC)) % 16 == 0);
  if (row < p.m && aux_vec && col0 + 32 <= p.n) {
#pragma unroll
    for (int j = 0; j < 32; j += 8) {
      const uint4 v = *reinterpret_cast<const uint4*>(aux + j);
      const TC* e = reinterpret_cast<const TC*>(&v);
#pragma unroll
      for (int t = 0; t < 8; ++t) u[j + t] = DT<TC>::to_f(e[t]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) u[j] = (row < p.m && col0 + j < p.n) ? DT<TC>::to_f(aux[j]) : 0.f;
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const float da = DT<TC>::to_f(DT<TC>::from_f(__uint_as_float(r[j])));
    r[j] = __float_as_uint(da * gelu_tanh_grad_f(u[j]));
  }
}

__device__ __forceinline__ void tile_coords(int t, const Params& p, int& mb, int& nb) {
  const int per_group = p.group_m * p.tiles_n;
  const int g = t / per_group;
  const int first_m = g * p.group_m;
  const int gm = min(p.group_m, p.tiles_m - first_m);
  const int r = t - g * per_group;
  mb = first_m + r % gm;
  nb = r / gm;
}

// One epilogue warp's share of one accumulator tile: TMEM lanes q*32 .. q*32+31
// (output rows row0 + q*32 + lane) and half `half` of the BN columns, read 32
// columns at a time from `tbase` (this warp's lane quarter, the tile's buffer) and
// written as f32 split-K partials, through the TMA staging slots (16-bit C, with
// the fused activation epilogues) or with direct row stores.
template <int BN, typename TC, int EPI>
__device__ __forceinline__ void epilogue_tile(const Params& p, uint8_t* stg, const CUtensorMap* tma_c,
                                              const CUtensorMap* tma_aux, uint32_t tbase, int row0, int nb,
                                              int split, int ew, int lane, int q, int half, bool vec_ok,
                                              bool ws_vec_ok, int& stg_count) {
  TC* c = reinterpret_cast<TC*>(p.c);
  const int row = row0 + q * 32 + lane;
#pragma unroll 1
  for (int cc = half * (BN / 64); cc < (half + 1) * (BN / 64); ++cc) {
    uint32_t r[32];
    tmem_ld32(tbase + cc * 32, r);
    tmem_wait_ld();
    if (p.splits > 1) {
      store_row32<float>(p.ws + (int64_t)split * p.m * p.n, p.n, row, nb * BN + cc * 32, p.m, p.n, r,
                         ws_vec_ok);
    } else if constexpr (sizeof(TC) == 2) {
      if (p.tma_store) {
        // this warp's 32 rows x 32 columns through a staging slot and one TMA
        // store (the unit clips rows / columns past M / N)
        const int x = nb * BN + cc * 32, y = row0 + q * 32;
        if constexpr (EPI == kEpiGeluBwd) epilogue_gelu_bwd_vals<TC>(p, row, x, r);
        stage_store_32x32<TC>(stg, ew, stg_count++, lane, r, tma_c, x, y);
        if constexpr (EPI == kEpiGelu) {
          uint32_t a[32];
#pragma unroll
          for (int j = 0; j < 32; ++j)
            a[j] = __float_as_uint(gelu_tanh_f(DT<TC>::to_f(DT<TC>::from_f(__uint_as_float(r[j])))));
          stage_store_32x32<TC>(stg, ew, stg_count++, lane, a, tma_aux, x, y);
        }
      } else {
        epilogue_row32<TC, EPI>(p, c, row, nb * BN + cc * 32, r, vec_ok);
      }
    } else {
      epilogue_row32<TC, EPI>(p, c, row, nb * BN + cc * 32, r, vec_ok);
    }
  }
}

// A_MN: A stored [K][M] (MN-major); B_MN: B stored [K][N] (MN-major).
template <int BN, bool A_MN, bool B_MN, bool BF16, typename TC, int EPI = kEpiNone>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tma_a,
                   const __grid_constant__ CUtensorMap tma_b,
                   const __grid_constant__ CUtensorMap tma_c,
                   const __grid_constant__ CUtensorMap tma_aux, const Params p) {
  using S = Smem<BN>;
  constexpr int STAGES = S::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* tiles = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_tiles = p.tiles_m * p.tiles_n;
  // Work unit u: tile u % num_tiles, K slice u / num_tiles (units of one slice
  // share a K range, so concurrently running CTAs share A/B rows in L2).
  const int num_units = num_tiles * p.splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kEpiWarps);  // one arrival per epilogue warp
    }
    *abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // PDL: every CTA holds its TMEM before the next kernel may be scheduled; no
  // global memory is touched before the previous kernel has completed.
  pdl_launch_dependents();
  pdl_wait();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
        int mb, nb;
        tile_coords(u % num_tiles, p, mb, nb);
        const int kb0 = (u / num_tiles) * p.kb_per_split;
        const int kb1 = min(kb0 + p.kb_per_split, p.k_blocks);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, abort, 1)) {
            ok = false;
            break;
          }
          uint8_t* sa = tiles + s * S::kStageBytes;
          uint8_t* sb = sa + S::kABytes;
          mbar_arrive_expect_tx(&full[s], S::kStageBytes);
          if constexpr (A_MN) {
            tma_load_2d(sa, &tma_a, &full[s], mb * BM, kb * BK);
            tma_load_2d(sa + 8192, &tma_a, &full[s], mb * BM + 64, kb * BK);
          } else {
            tma_load_2d(sa, &tma_a, &full[s], kb * BK, mb * BM);
          }
          if constexpr (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(sb + j * 8192, &tma_b, &full[s], nb * BN + j * 64, kb * BK);
          } else {
            tma_load_2d(sb, &tma_b, &full[s], kb * BK, nb * BN);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_f16(BM, BN, BF16, A_MN, B_MN);
      int it = 0, local = 0;
      bool ok = true;
      // Descriptors are built once; each MMA adds a byte offset (stage + K step).
      const uint32_t s0 = smem_u32(tiles);
      const uint64_t da_base = A_MN ? make_sdesc(s0, 8192, 1024) : make_sdesc(s0, 16, 1024);
      const uint64_t db_base = B_MN ? make_sdesc(s0 + S::kABytes, 8192, 1024)
                                    : make_sdesc(s0 + S::kABytes, 16, 1024);
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x, ++local) {
        const int buf = local & 1;
        const uint32_t aph = (local >> 1) & 1;
        if (!mbar_wait(&acc_empty[buf], aph ^ 1, abort, 2)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        const int kb0 = (u / num_tiles) * p.kb_per_split;
        const int kb1 = min(kb0 + p.kb_per_split, p.k_blocks);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&full[s], ph, abort, 3)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = sdesc_at(da_base, s * S::kStageBytes);
          const uint64_t db = sdesc_at(db_base, s * S::kStageBytes);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            tc_mma_f16_ss(d_tmem, sdesc_at(da, A_MN ? kk * 2048 : kk * 32),
                          sdesc_at(db, B_MN ? kk * 2048 : kk * 32), idesc,
                          (kb != kb0 || kk != 0) ? 1u : 0u);
          tc_commit(&empty[s]);  // slot free once these MMAs retire
        }
        tc_commit(&acc_full[buf]);  // accumulator ready for the epilogue
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;  // which half of the tile's columns
    const bool vec_ok = ((reinterpret_cast<uintptr_t>(p.c) & 15u) == 0) &&
                        ((p.ldc * (int64_t)sizeof(TC)) % 16 == 0);
    // partial slices are [m][n] f32 blocks of a 256-byte aligned workspace
    const bool ws_vec_ok = (p.n % 4 == 0);
    int stg_count = 0;  // staging slot use counter (slot = count & 1)
    int local = 0;
    for (int u = blockIdx.x; u < num_units; u += gridDim.x, ++local) {
      int mb, nb;
      tile_coords(u % num_tiles, p, mb, nb);
      const int split = u / num_tiles;
      const int buf = local & 1;
      const uint32_t aph = (local >> 1) & 1;
      if (!mbar_wait(&acc_full[buf], aph, abort, 4)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + buf * BN;
      epilogue_tile<BN, TC, EPI>(p, smem + S::kStgOff, &tma_c, &tma_aux, tbase, mb * BM, nb, split, warp - 2,
                                 lane, q, half, vec_ok, ws_vec_ok, stg_count);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
    if (lane == 0) bulk_wait_group0();  // this warp's TMA stores complete before exit
  }

  // ------------------------------------------------------------ teardown
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
  }
}

// ---------------------------------------------------------------------------
// CTA-pair variant: a cluster of two CTAs on two SMs computes one
// 256 x BN output tile with tcgen05.mma.cta_group::2 (M = 256).  Each CTA stages
// its own 128 rows of A and its own BN/2 columns of B, so per SM a 128 x BN x 64
// block of MMA work reads 16 KiB of A and BN*64 bytes of B from shared memory
// (and from L2) instead of 16 KiB + BN*128 bytes: B's shared-memory and L2
// traffic per FLOP halves, and the smaller stage leaves room for more stages.
//   * both CTAs' warp 0 issue TMA loads (no multicast) into their own shared
//     memory at the same offsets; the loads complete on the leader's (rank 0)
//     "full" barrier, which expects the bytes of both CTAs;
//   * the leader's warp 1 issues the pair MMAs; each MMA reads both CTAs'
//     operand halves and writes rows 0-127 of the accumulator into the leader's
//     TMEM and rows 128-255 into the peer's; its commits arrive on the "empty"
//     and "accumulator full" barriers of both CTAs;
//   * each CTA's epilogue drains its own TMEM rows and arrives on the leader's
//     "accumulator empty" barrier (16 arrivals: 8 warps per CTA);
//   * TMEM is allocated and freed by warp 1 of both CTAs together
//     (cta_group::2); the clusters synchronise after set-up and before
//     teardown, and each producer waits for the last release of every stage
//     before its CTA may leave, so no arrival targets a CTA that has exited.
// Every wait is bounded (kWaitLimitNs); an expired wait raises this CTA's abort
// flag, and the peer's waits expire within the same bound.
template <int BN>
struct Smem2 {
  static constexpr int kStages = BN == 256 ? 6 : 8;
  static constexpr int kABytes = BM * BK * 2;         // this CTA's 128 rows of A: 16 KiB
  static constexpr int kBBytes = (BN / 2) * BK * 2;   // this CTA's BN/2 columns of B
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTileBytes = kStages * kStageBytes;
  static constexpr int kSlotBytes = 32 * 32 * 2;
  static constexpr int kStgOff = kTileBytes;
  static constexpr int kStgBytes = kEpiWarps * 2 * kSlotBytes;
  static constexpr int kBarOff = kStgOff + kStgBytes;
  static constexpr int kBarBytes = (2 * kStages + 4) * 8 + 16;
  static constexpr int kTotal = 1024 + kBarOff + kBarBytes;
  static_assert(kTotal <= 227 * 1024, "shared memory per CTA");
};

template <int BN, bool A_MN, bool B_MN, bool BF16, typename TC, int EPI = kEpiNone>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tma_a,
                    const __grid_constant__ CUtensorMap tma_b,
                    const __grid_constant__ CUtensorMap tma_c,
                    const __grid_constant__ CUtensorMap tma_aux, const Params p) {
  using S = Smem2<BN>;
  constexpr int STAGES = S::kStages;
  constexpr int BM2 = 2 * BM;  // rows of a pair tile
  extern __shared__ uint8_t smem_raw[];
  // Same kernel, same shared-memory size: the aligned base (and so every stage)
  // sits at the same offset in both CTAs, as the pair MMA requires.
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* tiles = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0: the leader, which issues the MMAs
  const int pair = (int)(blockIdx.x >> 1);
  const int num_pairs = (int)(gridDim.x >> 1);
  const int num_tiles = p.tiles_m * p.tiles_n;  // pair tiles of 256 x BN
  // Work unit u: tile u % num_tiles, K slice u / num_tiles (as in the one-CTA kernel).
  const int num_units = num_tiles * p.splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);   // the leader's expect_tx arrival (+ both CTAs' bytes)
      mbar_init(&empty[s], 1);  // the leader's MMA commit
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2 * kEpiWarps);  // every epilogue warp of both CTAs
    }
    *abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 2 * BN);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers initialised and TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_launch_dependents();
  pdl_wait();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      const uint32_t full_leader = mapa_shared(full, 0);
      int it = 0;
      bool ok = true;
      for (int u = pair; u < num_units && ok; u += num_pairs) {
        int mb, nb;
        tile_coords(u % num_tiles, p, mb, nb);
        const int row = mb * BM2 + (int)rank * BM;         // this CTA's rows of A
        const int col = nb * BN + (int)rank * (BN / 2);    // this CTA's columns of B
        const int kb0 = (u / num_tiles) * p.kb_per_split;
        const int kb1 = min(kb0 + p.kb_per_split, p.k_blocks);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, abort, 1)) {
            ok = false;
            break;
          }
          uint8_t* sa = tiles + s * S::kStageBytes;
          uint8_t* sb = sa + S::kABytes;
          const uint32_t fb = full_leader + s * 8;
          if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * S::kStageBytes);
          if constexpr (A_MN) {
            tma_load_2d_pair(sa, &tma_a, fb, row, kb * BK);
            tma_load_2d_pair(sa + 8192, &tma_a, fb, row + 64, kb * BK);
          } else {
            tma_load_2d_pair(sa, &tma_a, fb, kb * BK, row);
          }
          if constexpr (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 128; ++j)
              tma_load_2d_pair(sb + j * 8192, &tma_b, fb, col + j * 64, kb * BK);
          } else {
            tma_load_2d_pair(sb, &tma_b, fb, kb * BK, col);
          }
        }
      }
      // Tail: the release of every stage's last use (the leader's commit, which
      // arrives on this CTA's barrier) has landed before this CTA may leave.
      for (int j = it; ok && j < it + STAGES; ++j)
        if (j >= STAGES && !mbar_wait(&empty[j % STAGES], ((j / STAGES) & 1) ^ 1, abort, 5)) ok = false;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader)
    if (rank == 0 && lane == 0) {
      constexpr uint32_t idesc = make_idesc_f16(BM2, BN, BF16, A_MN, B_MN);
      int it = 0, local = 0;
      bool ok = true;
      const uint32_t s0 = smem_u32(tiles);
      const uint64_t da_base = A_MN ? make_sdesc(s0, 8192, 1024) : make_sdesc(s0, 16, 1024);
      const uint64_t db_base = B_MN ? make_sdesc(s0 + S::kABytes, 8192, 1024)
                                    : make_sdesc(s0 + S::kABytes, 16, 1024);
      for (int u = pair; u < num_units && ok; u += num_pairs, ++local) {
        const int buf = local & 1;
        const uint32_t aph = (local >> 1) & 1;
        if (!mbar_wait(&acc_empty[buf], aph ^ 1, abort, 2)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        const int kb0 = (u / num_tiles) * p.kb_per_split;
        const int kb1 = min(kb0 + p.kb_per_split, p.k_blocks);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&full[s], ph, abort, 3)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = sdesc_at(da_base, s * S::kStageBytes);
          const uint64_t db = sdesc_at(db_base, s * S::kStageBytes);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            tc_mma_pair_ss(d_tmem, sdesc_at(da, A_MN ? kk * 2048 : kk * 32),
                           sdesc_at(db, B_MN ? kk * 2048 : kk * 32), idesc,
                           (kb != kb0 || kk != 0) ? 1u : 0u);
          tc_commit_pair(&empty[s], 0x3);  // both CTAs' slots free once these MMAs retire
        }
        if (ok) tc_commit_pair(&acc_full[buf], 0x3);  // both accumulator halves ready
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const bool vec_ok = ((reinterpret_cast<uintptr_t>(p.c) & 15u) == 0) &&
                        ((p.ldc * (int64_t)sizeof(TC)) % 16 == 0);
    const bool ws_vec_ok = (p.n % 4 == 0);
    const uint32_t acc_empty_leader = mapa_shared(acc_empty, 0);
    int stg_count = 0;
    int local = 0;
    for (int u = pair; u < num_units; u += num_pairs, ++local) {
      int mb, nb;
      tile_coords(u % num_tiles, p, mb, nb);
      const int buf = local & 1;
      const uint32_t aph = (local >> 1) & 1;
      if (!mbar_wait(&acc_full[buf], aph, abort, 4)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + buf * BN;
      epilogue_tile<BN, TC, EPI>(p, smem + S::kStgOff, &tma_c, &tma_aux, tbase, mb * BM2 + (int)rank * BM, nb,
                                 u / num_tiles, warp - 2, lane, q, half, vec_ok, ws_vec_ok, stg_count);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty_leader + buf * 8);
    }
    if (lane == 0) bulk_wait_group0();
  }

  // ------------------------------------------------------------ teardown
  tc_fence_before();
  __syncwarp();        // the warp reconverges before the aligned cluster barrier
  cluster_sync_all();  // both CTAs done with TMEM, shared memory and each other's barriers
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 2 * BN);
  }
}

// Split-K reduction: C = sum over slices (in slice order) of the f32 partials,
// rounded once to TC.  Four columns per thread (16-byte loads when n % 4 == 0).
template <typename TC>
__global__ void __launch_bounds__(256)
    splitk_reduce_kernel(const float* __restrict__ ws, TC* __restrict__ c, int m, int n,
                         int64_t ldc, int splits) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t plane = (int64_t)m * n;
  const int groups = (n + 3) / 4;
  const int64_t total = (int64_t)m * groups;
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total;
       g += (int64_t)gridDim.x * blockDim.x) {
    const int row = (int)(g / groups);
    const int col = (int)(g - (int64_t)row * groups) * 4;
    const float* src = ws + (int64_t)row * n + col;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    if (n % 4 == 0) {
      for (int sp = 0; sp < splits; ++sp) {
        const float4 v = __ldcs(reinterpret_cast<const float4*>(src + sp * plane));
        acc[0] += v.x;
        acc[1] += v.y;
        acc[2] += v.z;
        acc[3] += v.w;
      }
    } else {
      for (int sp = 0; sp < splits; ++sp)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (col + j < n) acc[j] += src[sp * plane + j];
    }
    TC* dst = c + (int64_t)row * ldc + col;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (col + j < n) dst[j] = DT<TC>::from_f(acc[j]);
  }
}

// ---------------------------------------------------------------------------
// CUDA-core path: exact f32 accumulation, any strides / transposes / dtypes.
// 128x128 CTA tile, 256 threads, 8x8 register micro-tile, K step 16.
// ---------------------------------------------------------------------------

constexpr int SB_M = 128, SB_N = 128, SB_K = 16;

template <typename TA>
__device__ __forceinline__ float ld_elem(const TA* p, int64_t idx) {
  return DT<TA>::to_f(p[idx]);
}

template <typename TA, typename TC>
__global__ void __launch_bounds__(256)
    gemm_simt_kernel(const TA* __restrict__ a, const TA* __restrict__ b, TC* __restrict__ c,
                     int m, int n, int k, int64_t lda, int64_t ldb, int64_t ldc,
                     int trans_a, int trans_b) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float As[2][SB_K][SB_M + 4];
  __shared__ float Bs[2][SB_K][SB_N + 4];
  const int tid = threadIdx.x;
  const int m0 = blockIdx.y * SB_M, n0 = blockIdx.x * SB_N;
  const int tr = tid / 16, tc = tid % 16;  // 16 x 16 threads, 8x8 each

  auto load_tile = [&](int buf, int k0) {
    // A tile: SB_M x SB_K elements = 2048, 8 per thread.
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = tid + i * 256;
      int mm, kk;
      if (trans_a) {  // stored [K][M]: consecutive threads along M
        mm = e % SB_M;
        kk = e / SB_M;
      } else {  // stored [M][K]: consecutive threads along K
        kk = e % SB_K;
        mm = e / SB_K;
      }
      const int gm = m0 + mm, gk = k0 + kk;
      float v = 0.f;
      if (gm < m && gk < k)
        v = ld_elem(a, trans_a ? (int64_t)gk * lda + gm : (int64_t)gm * lda + gk);
      As[buf][kk][mm] = v;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = tid + i * 256;
      int nn, kk;
      if (trans_b) {  // stored [N][K]
        kk = e % SB_K;
        nn = e / SB_K;
      } else {  // stored [K][N]
        nn = e % SB_N;
        kk = e / SB_N;
      }
      const int gn = n0 + nn, gk = k0 + kk;
      float v = 0.f;
      if (gn < n && gk < k)
        v = ld_elem(b, trans_b ? (int64_t)gn * ldb + gk : (int64_t)gk * ldb + gn);
      Bs[buf][kk][nn] = v;
    }
  };

  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  const int kt = (k + SB_K - 1) / SB_K;
  load_tile(0, 0);
  __syncthreads();
  for (int t = 0; t < kt; ++t) {
    const int cur = t & 1;
    if (t + 1 < kt) load_tile(cur ^ 1, (t + 1) * SB_K);
#pragma unroll
    for (int kk = 0; kk < SB_K; ++kk) {
      float av[8], bv[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        av[i] = As[cur][kk][tr * 4 + i];
        av[4 + i] = As[cur][kk][64 + tr * 4 + i];
        bv[i] = Bs[cur][kk][tc * 4 + i];
        bv[4 + i] = Bs[cur][kk][64 + tc * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int gm = m0 + (i < 4 ? tr * 4 + i : 64 + tr * 4 + (i - 4));
    if (gm >= m) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int gn = n0 + (j < 4 ? tc * 4 + j : 64 + tc * 4 + (j - 4));
      if (gn < n) c[(int64_t)gm * ldc + gn] = DT<TC>::from_f(acc[i][j]);
    }
  }
}

constexpr int kSkinnyM = 16;  // rows of A up to which the skinny kernel runs

// ---------------------------------------------------------------------------
// Skinny products, at most 16 rows of A (below the tensor-core path's 128-row tiles,
// which would be 16x redundant at 8 rows): the decode step's linears, y = x W with x
// [m <= 16, K] and W stored [K][N] row-major, and the tied LM head of decode and
// prefill, y = h E^T with E stored [N][K] (trans_b).  The cost is reading W once, and
// at these sizes (2-8 MB per layer matrix) nearly all of W has to be in flight at
// once.  A cluster of `cs` CTAs owns 64 output columns and splits K between its CTAs;
// each CTA streams its slice of the 64-column strip through a two-stage shared-memory
// ring with 16-byte cp.async copies (32 KB per stage: two stages hold the CTA's whole
// slice for K / cs <= 512), the 16-byte chunks of a row XOR-swizzled by the row
// index.  The products run on mma.sync m16n8k16 with the roles turned around,
// y^T = W^T x^T: W^T is the 16 x 16 A operand (ldmatrix.trans straight from [K][N]
// rows, plain ldmatrix from [N][K] rows; conflict-free thanks to the swizzle), x^T
// the 16 x 8 B operand (x kept 16-bit in shared memory, rows padded by 16 bytes),
// f32 accumulators.  The arithmetic is negligible either way; one MMA
// replaces 2048 FFMAs plus their conversions and shared-memory reads, which on CUDA
// cores made these launches issue-bound.  Warps take interleaved 16-row steps; the
// CTA sums its warps' tiles in shared memory, and the cluster's CTAs sum the partial
// tiles through distributed shared memory in rank order, each CTA writing its share
// of the outputs.  Fixed summation order (deterministic), no global scratch, one
// launch.
// ---------------------------------------------------------------------------
constexpr int kKnTileN = 64;
constexpr int kKnThreads = 256;
constexpr int kKnWarps = kKnThreads / 32;
constexpr int kKnStageRows = 256;  // rows of W per ring stage: 256 x 128 bytes
constexpr int kKnStages = 2;
constexpr int kKnMaxCluster = 8;
constexpr int kKnMaxSmem = 160 * 1024;
constexpr int kKnRowGrain = 64;  // rows per CTA are a multiple of this
constexpr int kKnAUnits = 4;     // 16-byte units of x loaded per thread before they are stored

// Shared memory of one CTA: the ring of W stages; x's rows [MR][kper + 8] (16-bit,
// padded so that the eight rows of an MMA operand fall in distinct banks); the warps'
// partial tiles [kKnWarps][MR][64] f32; the CTA's partial tile [MR][64] f32 that the
// cluster reads.
constexpr int kKnRingBytes = kKnStages * kKnStageRows * kKnTileN * 2;
__host__ __device__ constexpr int kn_x_bytes(int kper, int mr) { return (mr * (kper + 8) * 2 + 15) / 16 * 16; }
__host__ __device__ constexpr int kn_smem_bytes(int kper, int mr) {
  return 1024 /*alignment slack*/ + kKnRingBytes + kn_x_bytes(kper, mr) + (kKnWarps + 1) * mr * kKnTileN * 4;
}

__device__ __forceinline__ uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ float ld_shared_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}
// 16-byte global -> shared asynchronous copy, L2 only; src_bytes = 0 fills zeros.
__device__ __forceinline__ void cp_async16_zfill(void* smem, const void* gmem, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit_group() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
// Four 8 x 8 16-bit matrices, transposed on the way (lane L gives the address of row
// L % 8 of matrix L / 8).
__device__ __forceinline__ void ldmatrix_x4_trans(const void* p, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldmatrix_x4(const void* p, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
// d += a b, m16n8k16, 16-bit operands (A row-major, B column-major), f32 accumulators.
template <typename TA>
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  if constexpr (std::is_same<TA, __nv_bfloat16>::value)
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
                 "{%0, %1, %2, %3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
  else
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
                 "{%0, %1, %2, %3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// EPI: kEpiNone (C = acc) or kEpiGelu (C = u = round(acc), aux = round(gelu_tanh(u))).
// BNK: B stored [N][K] (trans_b) instead of [K][N]: a stage then holds the strip's 64
// rows of N, kKnStageRows elements of K each, as four 64-element column blocks of 128-byte
// rows (chunks swizzled by the row), and the W^T operand loads without the transpose.
// TMA: stages arrive as 2-D tiled TMA copies (128-byte swizzle, which is the chunk ^
// row % 8 layout above) completing on one mbarrier per stage -- a handful of
// instructions per stage and no per-SM limit on 16-byte copies in flight; else as
// 16-byte cp.async copies (shapes smaller than a TMA box).
// NORM: A is the normalised sum of two rows, the decode step's residual-add + RMSNorm
// folded in front of its product (rmsnorm.py:52-56 of the reference): h = x + r in f32,
// y = round(h * rsqrt(mean(h^2) + eps) * w) is the MMA operand.  Every CTA reads the
// whole rows (at most 16 x K, from L2) for the statistics, one warp per row in a fixed
// order, then stages its own K slice of y; CTA 0 alone writes round(h) to h_out.
struct KnNorm {
  const void* r;    // residual rows (row stride lda), or null: h = x
  const float* w;   // norm weight [K]
  void* h_out;      // round(h) (row stride lda), or null; never overlaps x or r
  float eps;
};

template <typename TA, typename TC, int MR, int EPI, bool BNK, bool TMA, bool NORM = false>
__global__ void __launch_bounds__(kKnThreads, 2)
    gemm_skinny_kn_kernel(const TA* __restrict__ a, const TA* __restrict__ b, TC* __restrict__ c, int m,
                          int n, int k, int kper, int64_t lda, int64_t ldb, int64_t ldc, int a_vec,
                          TC* __restrict__ aux, int64_t ld_aux, const __grid_constant__ CUtensorMap tmap_b,
                          int box_rows, const KnNorm nrm) {
  constexpr int NG = MR / 8;  // 8-row groups of x (MMA N = 8)
  extern __shared__ uint8_t kn_smem_raw[];
  // 1024-byte aligned base: the 128-byte swizzle pattern repeats every 1024 bytes
  uint8_t* kn_smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(kn_smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full_bar[kKnStages];
  __shared__ int abort_flag;
  volatile int* abort = &abort_flag;
  TA* ring = reinterpret_cast<TA*>(kn_smem);  // [kKnStages][kKnStageRows * 64], chunks swizzled
  TA* sx = reinterpret_cast<TA*>(kn_smem + kKnRingBytes);
  float* red = reinterpret_cast<float*>(kn_smem + kKnRingBytes + kn_x_bytes(kper, MR));
  float* part = red + kKnWarps * MR * kKnTileN;
  const int ldx = kper + 8;
  const int cs = (int)cluster_nctarank();
  const int rank = (int)cluster_ctarank();
  // persistent: cluster q takes the 64-column tiles q, q + clusters, ...; every CTA of
  // a cluster walks the same tiles, so the cluster barriers below pair up
  const int tiles = (n + kKnTileN - 1) / kKnTileN;
  const int cluster_id = (int)(blockIdx.x / cs), clusters = (int)(gridDim.x / cs);
  const int my_tiles = cluster_id < tiles ? (tiles - 1 - cluster_id) / clusters + 1 : 0;
  int col0 = cluster_id * kKnTileN;
  const int k0 = rank * kper;
  const int kn = max(0, min(k - k0, kper));  // rows of W this CTA reads
  const int nst = (kn + kKnStageRows - 1) / kKnStageRows;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tig = lane & 3;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    if constexpr (TMA) {
      mbar_init(&full_bar[0], 1);
      mbar_init(&full_bar[1], 1);
      fence_mbar_init();
      tma_prefetch_desc(&tmap_b);
    }
  }
  __syncthreads();
  pdl_launch_dependents();
  // Bring this CTA's strip of W into L2 while the previous kernel finishes (a launch
  // that follows through programmatic dependent launch starts early).  A prefetch
  // returns no data, so it is safe even if that kernel writes W: L2 keeps the newer lines.
  if constexpr (BNK) {
    if (kn > 0)  // one row of N per thread: kn elements of K (a multiple of 8)
      for (int r = threadIdx.x; r < kKnTileN && col0 + r < n; r += kKnThreads)
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(b + (int64_t)(col0 + r) * ldb + k0),
                     "r"((uint32_t)kn * 2)
                     : "memory");
  } else if (col0 < n) {
    const uint32_t bytes = (uint32_t)min(kKnTileN, n - col0) * 2;  // a multiple of 16
    for (int r = threadIdx.x; r < kn; r += kKnThreads)
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(b + (int64_t)(k0 + r) * ldb + col0), "r"(bytes)
                   : "memory");
  }
  pdl_wait();

  // stage st <- rows [bt * kKnStageRows, +kKnStageRows) of this CTA's slice of the
  // strip at column c0, 16 bytes (8 columns) per copy, chunk ch of row r at chunk
  // ch ^ (r % 8); rows past the slice and columns past n are zero-filled
  auto issue = [&](int st, int bt, int c0) {
    TA* dst = ring + st * kKnStageRows * kKnTileN;
    if constexpr (TMA) {
      // one thread: the stage's box(es); the barrier expects every byte they write
      // (zero fill past the tensor's edge included)
      if (threadIdx.x == 0) {
        if constexpr (BNK) {
          const int boxes = min(kKnStageRows / 64, (kn - bt * kKnStageRows + 63) / 64);
          mbar_arrive_expect_tx(&full_bar[st], (uint32_t)boxes * 64 * kKnTileN * 2);
          for (int j = 0; j < boxes; ++j)
            tma_load_2d(dst + j * 64 * kKnTileN, &tmap_b, &full_bar[st], k0 + bt * kKnStageRows + j * 64, c0);
        } else {
          mbar_arrive_expect_tx(&full_bar[st], (uint32_t)box_rows * kKnTileN * 2);
          tma_load_2d(dst, &tmap_b, &full_bar[st], c0, k0 + bt * box_rows);
        }
      }
      return;
    }
#pragma unroll
    for (int i = 0; i < kKnStageRows * 8 / kKnThreads; ++i) {
      const int ci = i * kKnThreads + threadIdx.x;
      if constexpr (BNK) {
        // row nl of the strip, chunk ch (8 elements of K) at chunk ch ^ (nl % 8);
        // kn % 8 == 0: a chunk is all in or all out
        const int nl = ci >> 5, ch = ci & 31;
        const int kk = bt * kKnStageRows + ch * 8;
        const bool ok = kk < kn && c0 + nl < n;
        const TA* src = ok ? b + (int64_t)(c0 + nl) * ldb + k0 + kk : b;
        cp_async16_zfill(dst + (ch >> 3) * 64 * kKnTileN + nl * 64 + (((ch & 7) ^ (nl & 7)) << 3), src, ok ? 16 : 0);
      } else {
        const int r = ci >> 3, ch = ci & 7;
        const int kk = bt * kKnStageRows + r, col = c0 + ch * 8;
        const bool ok = kk < kn && col < n;  // n % 8 == 0: a chunk is all in or all out
        const TA* src = ok ? b + (int64_t)(k0 + kk) * ldb + col : b;
        cp_async16_zfill(dst + r * kKnTileN + ((ch ^ (r & 7)) << 3), src, ok ? 16 : 0);
      }
    }
  };
  // the ring runs over the CTA's batches of all its tiles in one sequence: batch G is
  // batch G % nst of tile G / nst, in stage G % 2, issued two batches ahead, so the next
  // tile's copies fly while this tile is reduced
  const int total = my_tiles * nst;
  int issued = 0;  // batches whose copies were started (thread 0's count under TMA)
  auto issue_g = [&](int gb) {
    if (gb < total && !*abort) {
      issue(gb & 1, gb % nst, (cluster_id + (gb / nst) * clusters) * kKnTileN);
      issued = gb + 1;
    }
  };
  issue_g(0);
  if constexpr (!TMA) cp_async_commit_group();
  issue_g(1);
  if constexpr (!TMA) cp_async_commit_group();

  // NORM: per-row 1 / rms over the whole row of h (x + r), one warp per row; CTA 0
  // also writes round(h).  (k % 8 == 0 and 16-byte aligned rows: checked on the host.)
  __shared__ float s_inv[MR];
  if constexpr (NORM) {
    const TA* rr = static_cast<const TA*>(nrm.r);
    TA* ho = static_cast<TA*>(nrm.h_out);
    for (int row = warp; row < MR; row += kKnWarps) {
      float ss = 0.f;
      if (row < m) {
        for (int v = lane; v < k / 8; v += 32) {
          const uint4 xv = ld_v4(a + (int64_t)row * lda + v * 8);
          float h[8];
          const TA* xe = reinterpret_cast<const TA*>(&xv);
#pragma unroll
          for (int t = 0; t < 8; ++t) h[t] = DT<TA>::to_f(xe[t]);
          if (rr) {
            const uint4 rv = ld_v4(rr + (int64_t)row * lda + v * 8);
            const TA* re = reinterpret_cast<const TA*>(&rv);
#pragma unroll
            for (int t = 0; t < 8; ++t) h[t] += DT<TA>::to_f(re[t]);
          }
#pragma unroll
          for (int t = 0; t < 8; ++t) ss = fmaf(h[t], h[t], ss);
          if (ho && blockIdx.x == 0) {
            uint4 hv;
            TA* he = reinterpret_cast<TA*>(&hv);
#pragma unroll
            for (int t = 0; t < 8; ++t) he[t] = DT<TA>::from_f(h[t]);
            *reinterpret_cast<uint4*>(ho + (int64_t)row * lda + v * 8) = hv;
          }
        }
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
      if (lane == 0) s_inv[row] = rsqrtf(ss / (float)k + nrm.eps);
    }
    __syncthreads();
  }

  // x's rows [k0, k0 + kper) -> sx (zero past m and past kn); a pass issues all its
  // loads before its stores.  NORM: y's rows instead, from x, r and the weight.
  {
    const int vpr = kper / 8;
    const int units = MR * vpr;
    for (int base = 0; base < units; base += kKnThreads * kKnAUnits) {
      uint4 xv[kKnAUnits];
#pragma unroll
      for (int u = 0; u < kKnAUnits; ++u) {
        const int id = base + u * kKnThreads + threadIdx.x;
        const int r = id / vpr, kk = (id - r * vpr) * 8;
        const TA* src = a + (int64_t)r * lda + k0 + kk;
        if constexpr (NORM) {
          // kn % 8 == 0 here (k % 8 == 0, k0 a multiple of 64): whole vectors or none
          uint4 v = make_uint4(0u, 0u, 0u, 0u);
          if (id < units && r < m && kk < kn) {
            const uint4 x8 = ld_v4(src);
            const TA* xe = reinterpret_cast<const TA*>(&x8);
            float h[8];
#pragma unroll
            for (int t = 0; t < 8; ++t) h[t] = DT<TA>::to_f(xe[t]);
            if (nrm.r) {
              const uint4 r8 = ld_v4(static_cast<const TA*>(nrm.r) + (int64_t)r * lda + k0 + kk);
              const TA* re = reinterpret_cast<const TA*>(&r8);
#pragma unroll
              for (int t = 0; t < 8; ++t) h[t] += DT<TA>::to_f(re[t]);
            }
            const float4 w0 = *reinterpret_cast<const float4*>(nrm.w + k0 + kk);
            const float4 w1 = *reinterpret_cast<const float4*>(nrm.w + k0 + kk + 4);
            const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
            const float inv = s_inv[r];
            TA* ye = reinterpret_cast<TA*>(&v);
#pragma unroll
            for (int t = 0; t < 8; ++t) ye[t] = DT<TA>::from_f(h[t] * inv * wv[t]);
          }
          xv[u] = v;
        } else if (id < units && r < m && a_vec && kk + 8 <= kn) {
          xv[u] = ld_v4(src);
        } else {
          uint4 v;
          TA* e = reinterpret_cast<TA*>(&v);
#pragma unroll
          for (int t = 0; t < 8; ++t) e[t] = (id < units && r < m && kk + t < kn) ? src[t] : DT<TA>::from_f(0.f);
          xv[u] = v;
        }
      }
#pragma unroll
      for (int u = 0; u < kKnAUnits; ++u) {
        const int id = base + u * kKnThreads + threadIdx.x;
        const int r = id / vpr, kk = (id - r * vpr) * 8;
        if (id < units) *reinterpret_cast<uint4*>(sx + r * ldx + kk) = xv[u];
      }
    }
  }

  int gb = 0;  // batches consumed
  for (int tl = 0; tl < my_tiles; ++tl, col0 += clusters * kKnTileN) {
    float acc[4][NG][4];
#pragma unroll
    for (int s4 = 0; s4 < 4; ++s4)
#pragma unroll
      for (int ng = 0; ng < NG; ++ng)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[s4][ng][e] = 0.f;
    for (int bt = 0; bt < nst; ++bt, ++gb) {
      bool landed = true;
      if constexpr (TMA) {
        landed = !*abort && mbar_wait(&full_bar[gb & 1], (uint32_t)(gb >> 1) & 1u, abort, 130);
      } else {
        cp_async_wait_1();  // this stage's group has landed (the newest may still fly)
      }
      __syncthreads();  // ... for every thread's copies, and x's rows are staged
      const TA* st = ring + (gb & 1) * kKnStageRows * kKnTileN;
      const int rows = landed ? min(kKnStageRows, kn - bt * kKnStageRows) : 0;
      for (int ks = warp; ks * 16 < rows; ks += kKnWarps) {
        const int kl = ks * 16;
        const int kx = bt * kKnStageRows + kl;
        uint32_t bx[NG][2];
#pragma unroll
        for (int ng = 0; ng < NG; ++ng) {
          const TA* xp = sx + (ng * 8 + g) * ldx + kx + tig * 2;
          bx[ng][0] = *reinterpret_cast<const uint32_t*>(xp);
          bx[ng][1] = *reinterpret_cast<const uint32_t*>(xp + 8);
        }
#pragma unroll
        for (int s4 = 0; s4 < 4; ++s4) {
          uint32_t wa[4];
          if constexpr (BNK) {
            // matrix q = lane / 8: rows of N s4*16 + (q & 1) * 8 + lane % 8, K chunk ks*2 + q / 2
            const int nl = s4 * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
            const int chunk = ks * 2 + (lane >> 4);  // 8-element chunk of the stage's K
            ldmatrix_x4(st + (chunk >> 3) * 64 * kKnTileN + nl * 64 + (((chunk & 7) ^ (nl & 7)) << 3), wa);
          } else {
            // matrix q = lane / 8: rows of K kl + (q / 2) * 8 + lane % 8, N chunk s4*2 + q % 2
            const int row = kl + (lane & 7) + ((lane >> 4) << 3);
            const int chunk = s4 * 2 + ((lane >> 3) & 1);
            ldmatrix_x4_trans(st + row * kKnTileN + ((chunk ^ (row & 7)) << 3), wa);
          }
#pragma unroll
          for (int ng = 0; ng < NG; ++ng) mma_16816<TA>(acc[s4][ng], wa, bx[ng]);
        }
      }
      __syncthreads();  // the stage is free again
      issue_g(gb + 2);
      if constexpr (!TMA) cp_async_commit_group();
    }

    // accumulator (W column n0 + g [+8], x row tig*2 + e) -> the warp's tile, then the
    // warps' tiles -> the CTA's partial tile
#pragma unroll
    for (int s4 = 0; s4 < 4; ++s4)
#pragma unroll
      for (int ng = 0; ng < NG; ++ng)
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int e = 0; e < 2; ++e)
            red[(warp * MR + ng * 8 + tig * 2 + e) * kKnTileN + s4 * 16 + g + h * 8] = acc[s4][ng][h * 2 + e];
    __syncthreads();
    for (int v = threadIdx.x; v < MR * kKnTileN; v += kKnThreads) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < kKnWarps; ++w) s += red[w * MR * kKnTileN + v];
      part[v] = s;
    }
    if (cs > 1) cluster_sync_all();  // every CTA's partial tile is visible to the cluster
    else __syncthreads();
    const int per = MR * kKnTileN / cs;  // cs is a power of two <= 8
    for (int v = rank * per + threadIdx.x; v < (rank + 1) * per; v += kKnThreads) {
      const int r = v / kKnTileN, cc = col0 + v % kKnTileN;
      if (r >= m || cc >= n) continue;
      float s = 0.f;
      for (int q = 0; q < cs; ++q) s += ld_shared_cluster_f32(mapa_shared(part + v, (uint32_t)q));
      const TC u = DT<TC>::from_f(s);
      c[(int64_t)r * ldc + cc] = u;
      if constexpr (EPI == kEpiGelu) aux[(int64_t)r * ld_aux + cc] = DT<TC>::from_f(gelu_tanh_f(DT<TC>::to_f(u)));
    }
    if (cs > 1) cluster_sync_all();  // no CTA rewrites (or leaves) its partial tile while another reads it
    else __syncthreads();
  }
  // after an expired wait: let the copies still in flight land (bounded) before the
  // shared memory they write is released.  No batch is issued after the abort, and at
  // most two are in flight at once: the last two issued (a wait on a phase that has
  // already completed returns at once).
  if constexpr (TMA) {
    if (threadIdx.x == 0 && *abort) {
      int never = 0;
      for (int q = max(0, issued - 2); q < issued; ++q)
        (void)mbar_wait_ns(&full_bar[q & 1], (uint32_t)(q >> 1) & 1u, &never, 131, kWaitLimitNs);
    }
  }
}

// ---------------------------------------------------------------------------
// host
// ---------------------------------------------------------------------------

static int env_int(const char* name, int dflt) {
  const char* s = std::getenv(name);
  return (s && *s) ? std::atoi(s) : dflt;
}

template <typename TA, typename TC>
static int launch_simt(cudaStream_t s, const void* a, const void* b, void* c, int64_t m,
                       int64_t n, int64_t k, int64_t lda, int64_t ldb, int64_t ldc,
                       int ta, int tb) {
  dim3 grid((unsigned)((n + SB_N - 1) / SB_N), (unsigned)((m + SB_M - 1) / SB_M));
  if (grid.y > 65535) return fail(FERRITE_BAD_SHAPE, "gemm: M too large for the CUDA-core path");
  (void)launch_pdl(gemm_simt_kernel<TA, TC>, dim3(grid), dim3(256), 0, s, (const TA*)a, (const TA*)b, (TC*)c, (int)m,
                                                 (int)n, (int)k, lda, ldb, ldc, ta, tb);
  return check_launch("gemm_simt");
}

// Clusters of two gemm_tc2_kernel CTAs resident at once on `dev` (cached per
// device; every instance has the same block size and shared memory, so one
// representative instance answers for all).
static int pair_slots(int dev, int sms) {
  static int cache[64] = {0};
  if (dev < 0 || dev >= 64) return sms / 2;
  if (cache[dev] == 0) {
    auto kern = gemm_tc2_kernel<256, false, false, true, __nv_bfloat16>;
    int n = 0;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Smem2<256>::kTotal) == cudaSuccess)
      n = max_active_clusters((const void*)kern, dim3(kThreads), Smem2<256>::kTotal, 2);
    else
      (void)cudaGetLastError();
    cache[dev] = n > 0 ? n : sms / 2;
  }
  return cache[dev];
}

// Cluster size and rows of K per CTA for the skinny path: K is split over a cluster
// (up to 8 CTAs) while the grid of 64-column tiles would not cover half the SMs and
// each CTA keeps at least one full stage of rows (below that the cluster's fixed costs
// win: 1024 x 1024 ran 6% faster on 4 CTAs than on 8), so that most of W is in flight
// at once; or while x's slice would not fit in shared memory.  Wide outputs (the LM head's 32000 columns) keep whole K per CTA and are
// covered by persistent clusters looping over their tiles.
struct KnPlan {
  int cs, kper, smem;
};
static KnPlan kn_plan(int64_t m, int64_t n, int64_t k, int sms) {
  const int mr = m <= 8 ? 8 : kSkinnyM;
  const int64_t tiles = (n + kKnTileN - 1) / kKnTileN;
  auto kper_for = [&](int c) {
    const int64_t rows = (k + c - 1) / c;
    return std::min<int64_t>((rows + kKnRowGrain - 1) / kKnRowGrain * kKnRowGrain, 1 << 20);
  };
  int cs = 1;
  while (cs < kKnMaxCluster) {
    const bool spread = tiles * cs * 2 <= sms && (k + 2 * cs - 1) / (2 * cs) >= kKnStageRows;
    const bool fits = kn_smem_bytes((int)kper_for(cs), mr) <= kKnMaxSmem;
    if (!spread && fits) break;
    cs *= 2;
  }
  const int kper = (int)kper_for(cs);
  return {cs, kper, kn_smem_bytes(kper, mr)};
}

// Skinny path: 16-bit operands, A K-major with at most kSkinnyM rows; B with 16-byte
// aligned rows (ldb a multiple of 8) stored [K][N] with N a multiple of 8, or [N][K]
// (trans_b) with K a multiple of 8 (16-byte copies never straddle the edge); K bounded
// by shared memory.
static bool skinny_kn_ok(const void* b, int64_t m, int64_t n, int64_t k, int64_t ldb, int trans_a,
                         int trans_b) {
  if (env_int("FERRITE_GEMM_SKINNY", 1) == 0) return false;
  if (trans_a || m < 1 || m > kSkinnyM || n < 1 || k < 1) return false;
  if (trans_b ? k % 8 != 0 : n % 8 != 0) return false;
  if ((reinterpret_cast<uintptr_t>(b) & 15u) || ldb % 8) return false;
  if (n > 0x7fffffff || k > 0x7fffffff) return false;
  return kn_plan(m, n, k, num_sms(current_device())).smem <= kKnMaxSmem;
}

// Clusters of `cs` CTAs of `kern` with `smem` bytes each that fit on the device at
// once (cached per kernel, cluster size, shared memory and device).
static int kn_cluster_slots(const void* kern, int cs, int smem) {
  struct Entry {
    const void* f;
    int cs, smem, dev, n;
  };
  static std::mutex mu;
  static Entry cache[64];
  static int used = 0;
  const int dev = current_device();
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; ++i)
    if (cache[i].f == kern && cache[i].cs == cs && cache[i].smem == smem && cache[i].dev == dev) return cache[i].n;
  int n = max_active_clusters(kern, dim3(kKnThreads), (size_t)smem, (unsigned)cs);
  if (n <= 0) {
    (void)cudaGetLastError();
    n = std::max(1, num_sms(dev) / cs);
  }
  if (used < 64) cache[used++] = {kern, cs, smem, dev, n};
  return n;
}

template <typename TA, typename TC, int EPI = kEpiNone, bool NORM = false>
static int launch_skinny_kn(cudaStream_t s, const void* a, const void* b, void* c, int64_t m, int64_t n,
                            int64_t k, int64_t lda, int64_t ldb, int64_t ldc, int trans_b,
                            void* aux = nullptr, int64_t ld_aux = 0, KnNorm nrm = KnNorm{nullptr, nullptr, nullptr, 0.f}) {
  const KnPlan pl = kn_plan(m, n, k, num_sms(current_device()));
  // TMA stages when every box fits inside the tensor: [K][N] boxes are 64 columns x
  // min(256, rows per CTA) rows, [N][K] boxes 64 x 64
  const int box_rows = std::min(kKnStageRows, pl.kper);
  const bool tma = trans_b ? (k >= 64 && n >= kKnTileN) : (n >= kKnTileN && k >= box_rows);
  using Kern = void (*)(const TA*, const TA*, TC*, int, int, int, int, int64_t, int64_t, int64_t, int, TC*, int64_t,
                        const CUtensorMap, int, const KnNorm);
  Kern kern;
  if (trans_b) {
    if (tma) kern = m <= 8 ? gemm_skinny_kn_kernel<TA, TC, 8, EPI, true, true, NORM> : gemm_skinny_kn_kernel<TA, TC, kSkinnyM, EPI, true, true, NORM>;
    else kern = m <= 8 ? gemm_skinny_kn_kernel<TA, TC, 8, EPI, true, false, NORM> : gemm_skinny_kn_kernel<TA, TC, kSkinnyM, EPI, true, false, NORM>;
  } else {
    if (tma) kern = m <= 8 ? gemm_skinny_kn_kernel<TA, TC, 8, EPI, false, true, NORM> : gemm_skinny_kn_kernel<TA, TC, kSkinnyM, EPI, false, true, NORM>;
    else kern = m <= 8 ? gemm_skinny_kn_kernel<TA, TC, 8, EPI, false, false, NORM> : gemm_skinny_kn_kernel<TA, TC, kSkinnyM, EPI, false, false, NORM>;
  }
  // (a runtime call first: it makes the device's primary context current on this
  // thread -- e.g. an autograd worker -- which the tensor-map encoder needs)
  {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, pl.smem);
    if (e != cudaSuccess) return fail(FERRITE_LAUNCH_FAILED, "gemm: skinny smem attribute: %s", cudaGetErrorString(e));
  }
  CUtensorMap tmap;
  std::memset(&tmap, 0, sizeof(tmap));
  if (tma) {
    const CUtensorMapDataType dt = std::is_same<TA, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                         : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const int rc = trans_b ? make_tmap_2d(&tmap, b, dt, 2, (uint64_t)k, (uint64_t)n, (uint64_t)ldb * 2, 64, kKnTileN,
                                          CU_TENSOR_MAP_SWIZZLE_128B)
                           : make_tmap_2d(&tmap, b, dt, 2, (uint64_t)n, (uint64_t)k, (uint64_t)ldb * 2, kKnTileN,
                                          (uint32_t)box_rows, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  // x's rows as 16-byte vectors: aligned base and row stride (kper, hence k0, is a multiple of 16)
  const int a_vec = (reinterpret_cast<uintptr_t>(a) & 15u) == 0 && lda % 8 == 0;
  // persistent clusters: at most as many as fit at once, each looping over its tiles
  const int64_t tiles = (n + kKnTileN - 1) / kKnTileN;
  const int64_t clusters = std::min<int64_t>(tiles, kn_cluster_slots((const void*)kern, pl.cs, pl.smem));
  (void)launch_pdl_cluster(kern, dim3((unsigned)(clusters * pl.cs)), dim3(kKnThreads), (size_t)pl.smem, s,
                           (unsigned)pl.cs, (const TA*)a, (const TA*)b, (TC*)c, (int)m, (int)n, (int)k,
                           pl.kper, lda, ldb, ldc, a_vec, (TC*)aux, ld_aux, tmap, box_rows, nrm);
  return check_launch("gemm_skinny_kn");
}

// PAIR: the CTA-pair kernel (grid: two CTAs per cluster, at most the clusters
// that fit at once); else the one-CTA kernel (grid: min(units, SMs)).
template <bool PAIR, int BN, bool A_MN, bool B_MN, bool BF16, typename TC, int EPI = kEpiNone>
static int launch_tc(cudaStream_t s, const CUtensorMap& ta, const CUtensorMap& tb,
                     const CUtensorMap& tc, const CUtensorMap& taux, const Params& p, int units, int sms) {
  if constexpr (PAIR) {
    auto kern = gemm_tc2_kernel<BN, A_MN, B_MN, BF16, TC, EPI>;
    const int smem = Smem2<BN>::kTotal;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess)
      return fail(FERRITE_LAUNCH_FAILED, "gemm: smem attribute: %s", cudaGetErrorString(e));
    const int clusters = std::min(units, pair_slots(current_device(), sms));
    (void)launch_pdl_cluster(kern, dim3(2 * clusters), dim3(kThreads), smem, s, 2u, ta, tb, tc, taux, p);
    return check_launch("gemm_tc2");
  } else {
    auto kern = gemm_tc_kernel<BN, A_MN, B_MN, BF16, TC, EPI>;
    const int smem = Smem<BN>::kTotal;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess)
      return fail(FERRITE_LAUNCH_FAILED, "gemm: smem attribute: %s", cudaGetErrorString(e));
    (void)launch_pdl(kern, dim3(std::min(units, sms)), dim3(kThreads), smem, s, ta, tb, tc, taux, p);
    return check_launch("gemm_tc");
  }
}

template <bool PAIR, int BN, bool BF16, typename TC>
static int dispatch_major(cudaStream_t s, bool a_mn, bool b_mn, const CUtensorMap& ta,
                          const CUtensorMap& tb, const CUtensorMap& tc, const CUtensorMap& taux,
                          const Params& p, int units, int sms, int epi) {
  if constexpr (BF16 && std::is_same<TC, __nv_bfloat16>::value) {
    // the GPT MLP's fused epilogues: up-projection (A K-major, B MN-major) and
    // dA = dP W2^T (both K-major)
    if (epi == kEpiGelu && !a_mn && b_mn)
      return launch_tc<PAIR, BN, false, true, true, TC, kEpiGelu>(s, ta, tb, tc, taux, p, units, sms);
    if (epi == kEpiGeluBwd && !a_mn && !b_mn)
      return launch_tc<PAIR, BN, false, false, true, TC, kEpiGeluBwd>(s, ta, tb, tc, taux, p, units, sms);
  }
  if (epi != kEpiNone)
    return fail(FERRITE_UNSUPPORTED_DTYPE, "gemm: epilogue %d needs bf16 operands and output with %s", epi,
                epi == kEpiGelu ? "A K-major, B [K][N]" : "A K-major, B [N][K] (trans_b)");
  if (!a_mn && !b_mn) return launch_tc<PAIR, BN, false, false, BF16, TC>(s, ta, tb, tc, taux, p, units, sms);
  if (!a_mn && b_mn) return launch_tc<PAIR, BN, false, true, BF16, TC>(s, ta, tb, tc, taux, p, units, sms);
  if (a_mn && !b_mn) return launch_tc<PAIR, BN, true, false, BF16, TC>(s, ta, tb, tc, taux, p, units, sms);
  return launch_tc<PAIR, BN, true, true, BF16, TC>(s, ta, tb, tc, taux, p, units, sms);
}

// Tile shape and K split.  Cost model in units of one 128x256x64 MMA block on
// one SM: a 128-wide tile block costs 0.69 (half the FLOPs at ~72% of the
// 256-wide rate, measured) and a block of a CTA-pair tile 0.95 (the pair kernel
// ran 5% faster than the one-CTA kernel on 8192^3); waves are ceil(units /
// slots) with one slot per SM (one-CTA tiles) or per resident cluster of two
// (pair tiles, 256 rows each); a split adds the f32 partial traffic (write +
// read of splits x M x N x 4 bytes, ~2.3 MB per unit of time at HBM rate) plus
// the reduction launch.
struct Plan {
  int bn, splits, kb_per_split;
  bool pair;
};

static Plan plan_tc(int64_t m, int64_t n, int64_t k, int sms, int pair_slots, bool allow_split) {
  const int64_t kb = (k + BK - 1) / BK;
  Plan best{n < 256 ? 128 : 256, 1, (int)kb, false};
  double best_cost = 1e300;
  const int max_splits = allow_split ? (int)std::min<int64_t>(16, kb / 4) : 1;
  const bool pair_ok = pair_slots > 0 && m >= 2 * BM && n >= 256 && env_int("FERRITE_GEMM_PAIR", 1) != 0;
  struct Shape {
    bool pair;
    int bn;
    double unit;
  };
  const Shape shapes[3] = {{true, 256, 0.95}, {false, 256, 1.0}, {false, 128, 0.69}};
  for (const Shape& sh : shapes) {
    if (sh.pair && !pair_ok) continue;
    if (sh.bn == 256 && n < 256) continue;
    const int64_t rows = sh.pair ? 2 * BM : BM;
    const int64_t tiles = ((m + rows - 1) / rows) * ((n + sh.bn - 1) / sh.bn);
    const int64_t slots = sh.pair ? pair_slots : sms;
    for (int sp = 1; sp <= std::max(1, max_splits); ++sp) {
      const int64_t kbs = (kb + sp - 1) / sp;
      const int64_t eff_splits = (kb + kbs - 1) / kbs;  // no empty slices
      if (eff_splits != sp) continue;
      const int64_t units = tiles * sp;
      const double waves = (double)((units + slots - 1) / slots);
      double cost = waves * (double)kbs * sh.unit;
      if (sp > 1) cost += 2.0 * sp * (double)m * (double)n * 4.0 / 2.3e6 + 13.0;
      if (cost < best_cost * 0.97) {  // prefer the earlier shape / fewer splits on near-ties
        best_cost = cost;
        best = Plan{sh.bn, sp, (int)kbs, sh.pair};
      }
    }
  }
  const int forced = env_int("FERRITE_GEMM_BN", 0);
  if ((forced == 128 || forced == 256) && n >= forced) {
    best.bn = forced;
    if (forced == 128) best.pair = false;
  }
  const int forced_split = env_int("FERRITE_GEMM_SPLITS", 0);
  if (allow_split && forced_split >= 1) {
    const int64_t kbs = (kb + forced_split - 1) / forced_split;
    best.splits = (int)((kb + kbs - 1) / kbs);
    best.kb_per_split = (int)kbs;
  }
  if (env_int("FERRITE_GEMM_PAIR", -1) == 1 && pair_ok && best.bn == 256) best.pair = true;  // forced on
  return best;
}

static size_t plan_workspace(const Plan& pl, int64_t m, int64_t n) {
  return pl.splits > 1 ? (size_t)pl.splits * (size_t)m * (size_t)n * sizeof(float) : 0;
}

template <typename TC>
static int launch_reduce(cudaStream_t s, const float* ws, void* c, int64_t m, int64_t n,
                         int64_t ldc, int splits, int sms) {
  const int64_t groups = m * ((n + 3) / 4);
  const int64_t want = (groups + 255) / 256;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)sms * 8));
  (void)launch_pdl(splitk_reduce_kernel<TC>, dim3(grid), dim3(256), 0, s, ws, (TC*)c, (int)m, (int)n, ldc, splits);
  return check_launch("gemm_splitk_reduce");
}

template <bool BF16, typename TC>
static int run_tc(cudaStream_t s, const void* a, const void* b, void* c, int64_t m,
                  int64_t n, int64_t k, int64_t lda, int64_t ldb, int64_t ldc, int trans_a,
                  int trans_b, void* workspace, size_t ws_bytes, int epi = kEpiNone,
                  void* aux = nullptr, int64_t ld_aux = 0) {
  const int dev = current_device();
  const int sms = num_sms(dev);
  const int pslots = pair_slots(dev, sms);
  Plan pl = plan_tc(m, n, k, sms, pslots, workspace != nullptr && epi == kEpiNone);
  if (plan_workspace(pl, m, n) > ws_bytes || (reinterpret_cast<uintptr_t>(workspace) & 255u)) {
    pl = plan_tc(m, n, k, sms, pslots, false);  // not enough scratch: no split
  }
  const int BN = pl.bn;
  const bool pair = pl.pair;  // 256 x 256 tiles on CTA pairs (FERRITE_GEMM_PAIR=0: never)

  const CUtensorMapDataType dt = BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap ta, tb;
  const bool a_mn = trans_a != 0;  // A stored [K][M]
  const bool b_mn = trans_b == 0;  // B stored [K][N] is MN-major for the MMA
  int rc;
  if (a_mn)
    rc = make_tmap_2d(&ta, a, dt, 2, (uint64_t)m, (uint64_t)k, (uint64_t)lda * 2, 64, 64,
                      CU_TENSOR_MAP_SWIZZLE_128B);
  else
    rc = make_tmap_2d(&ta, a, dt, 2, (uint64_t)k, (uint64_t)m, (uint64_t)lda * 2, 64, 128,
                      CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  if (b_mn)
    rc = make_tmap_2d(&tb, b, dt, 2, (uint64_t)n, (uint64_t)k, (uint64_t)ldb * 2, 64, 64,
                      CU_TENSOR_MAP_SWIZZLE_128B);
  else
    rc = make_tmap_2d(&tb, b, dt, 2, (uint64_t)k, (uint64_t)n, (uint64_t)ldb * 2, 64,
                      (uint32_t)(pair ? BN / 2 : BN), CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;

  Params p;
  p.m = (int)m;
  p.n = (int)n;
  p.k = (int)k;
  p.ldc = ldc;
  p.c = c;
  const int64_t tile_rows = pair ? 2 * BM : BM;
  p.tiles_m = (int)((m + tile_rows - 1) / tile_rows);
  p.tiles_n = (int)((n + BN - 1) / BN);
  p.k_blocks = (int)((k + BK - 1) / BK);
  // Raster group: the A rows of one group span about 32 MiB of bf16 over the whole K
  // range (16 Mi elements), at most 16 tiles.  At 8192^3 that is 2048 rows: the group's
  // A stays L2-resident while its units sweep N, and the kernel ran 3% faster (at a
  // 3% higher clock under the power cap) than with 4096-row groups.
  const int64_t group_rows = std::max<int64_t>(tile_rows, (int64_t(16) << 20) / std::max<int64_t>(k, 1));
  const int gm_default = (int)std::min<int64_t>(16, std::max<int64_t>(1, group_rows / tile_rows));
  p.group_m = std::max(1, std::min(env_int("FERRITE_GEMM_GROUP_M", gm_default), p.tiles_m));
  p.splits = pl.splits;
  p.kb_per_split = pl.kb_per_split;
  p.ws = pl.splits > 1 ? reinterpret_cast<float*>(workspace) : nullptr;
  p.aux = aux;
  p.ld_aux = ld_aux;
  const int units = p.tiles_m * p.tiles_n * p.splits;
  // 16-bit C (and the GELU epilogue's aux output) through TMA stores: 32 x 32
  // boxes, 64-byte swizzle; a layout TMA cannot describe keeps direct stores
  CUtensorMap tc = ta, taux = ta;  // placeholders when unused (never dereferenced)
  p.tma_store = 0;
  if (sizeof(TC) == 2 && pl.splits == 1 && env_int("FERRITE_GEMM_TMA_STORE", 1)) {
    const CUtensorMapDataType ct = std::is_same<TC, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                         : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const bool c_ok = (reinterpret_cast<uintptr_t>(c) & 15u) == 0 && (ldc * 2) % 16 == 0;
    const bool aux_ok = epi != kEpiGelu || ((reinterpret_cast<uintptr_t>(aux) & 15u) == 0 && (ld_aux * 2) % 16 == 0);
    if (c_ok && aux_ok &&
        make_tmap_2d(&tc, c, ct, 2, (uint64_t)n, (uint64_t)m, (uint64_t)ldc * 2, 32, 32,
                     CU_TENSOR_MAP_SWIZZLE_64B) == FERRITE_OK &&
        (epi != kEpiGelu || make_tmap_2d(&taux, aux, ct, 2, (uint64_t)n, (uint64_t)m, (uint64_t)ld_aux * 2, 32, 32,
                                         CU_TENSOR_MAP_SWIZZLE_64B) == FERRITE_OK))
      p.tma_store = 1;
  }
  rc = pair        ? dispatch_major<true, 256, BF16, TC>(s, a_mn, b_mn, ta, tb, tc, taux, p, units, sms, epi)
       : BN == 256 ? dispatch_major<false, 256, BF16, TC>(s, a_mn, b_mn, ta, tb, tc, taux, p, units, sms, epi)
                   : dispatch_major<false, 128, BF16, TC>(s, a_mn, b_mn, ta, tb, tc, taux, p, units, sms, epi);
  if (rc || pl.splits == 1) return rc;
  return launch_reduce<TC>(s, p.ws, c, m, n, ldc, pl.splits, sms);
}

// True when every operand satisfies the TMA rules and the tile shapes fit.
static bool tc_eligible(const void* a, const void* b, int64_t m, int64_t n, int64_t k,
                        int64_t lda, int64_t ldb, int trans_a, int trans_b) {
  if (env_int("FERRITE_GEMM_FORCE_SIMT", 0)) return false;
  if ((reinterpret_cast<uintptr_t>(a) & 15u) || (reinterpret_cast<uintptr_t>(b) & 15u)) return false;
  if ((lda * 2) % 16 || (ldb * 2) % 16) return false;
  // Keep every TMA box inside the tensor extent along each dimension.
  if (m < BM || n < 128 || k < BK) return false;
  (void)trans_a;
  (void)trans_b;
  if (m > 0x7fffffff || n > 0x7fffffff || k > 0x7fffffff) return false;
  return true;
}

}  // namespace gemm
}  // namespace ferrite

using namespace ferrite;
using namespace ferrite::gemm;

extern "C" size_t ferrite_gemm_workspace_size(int64_t m, int64_t n, int64_t k, int64_t lda,
                                              int64_t ldb, int trans_a, int trans_b,
                                              int ab_dtype) {
  if (m <= 0 || n <= 0 || k <= 0 || ab_dtype == FERRITE_F32) return 0;
  if (m > 0x7fffffff || n > 0x7fffffff || k > 0x7fffffff) return 0;
  // Same eligibility rules as the launch, with aligned stand-in pointers.
  const void* aligned = reinterpret_cast<const void*>(uintptr_t(256));
  if (!tc_eligible(aligned, aligned, m, n, k, lda, ldb, trans_a, trans_b)) return 0;
  const int dev = current_device();
  const int sms = num_sms(dev);
  return plan_workspace(plan_tc(m, n, k, sms, pair_slots(dev, sms), true), m, n);
}

extern "C" int ferrite_gemm(void* stream, const void* a, const void* b, void* c, int64_t m,
                            int64_t n, int64_t k, int64_t lda, int64_t ldb, int64_t ldc,
                            int trans_a, int trans_b, int ab_dtype, int c_dtype) {
  return ferrite_gemm_ws(stream, a, b, c, m, n, k, lda, ldb, ldc, trans_a, trans_b, ab_dtype,
                         c_dtype, nullptr, 0);
}

// Residual-add + RMSNorm in front of a skinny product (the decode step): see the header.
extern "C" int ferrite_gemm_rmsnorm(void* stream, const void* x, const void* r, const float* w_norm, float eps,
                                    void* h_out, const void* b, void* c, int64_t m, int64_t n, int64_t k,
                                    int64_t ldx, int64_t ldb, int64_t ldc, int trans_b, int epilogue, void* aux,
                                    int64_t ld_aux, int ab_dtype, int c_dtype) {
  if (int rc = injected_fault("gemm")) return rc;
  if (m < 0 || n < 0 || k < 0) return fail(FERRITE_BAD_SHAPE, "gemm_rmsnorm: negative size");
  if (m == 0) return FERRITE_OK;
  if (m > kSkinnyM) return fail(FERRITE_BAD_SHAPE, "gemm_rmsnorm: at most %d rows, got %lld", kSkinnyM, (long long)m);
  if (n < 1 || k < 8 || k % 8) return fail(FERRITE_BAD_SHAPE, "gemm_rmsnorm: needs n >= 1 and k a positive multiple of 8");
  if (ab_dtype != FERRITE_BF16 && ab_dtype != FERRITE_F16)
    return fail(FERRITE_UNSUPPORTED_DTYPE, "gemm_rmsnorm: operands must be bf16 or f16");
  if (c_dtype != ab_dtype && c_dtype != FERRITE_F32)
    return fail(FERRITE_UNSUPPORTED_DTYPE, "gemm_rmsnorm: output dtype must be the operands' or f32");
  if (epilogue != kEpiNone && epilogue != kEpiGelu) return fail(FERRITE_BAD_SHAPE, "gemm_rmsnorm: unknown epilogue %d", epilogue);
  if (epilogue == kEpiGelu && (trans_b || ab_dtype != FERRITE_BF16 || c_dtype != FERRITE_BF16 || !aux || ld_aux < n))
    return fail(FERRITE_BAD_SHAPE, "gemm_rmsnorm: the GELU epilogue needs bf16, B stored [K][N] and aux [m][>= n]");
  if (!x || !w_norm || !b || !c) return fail(FERRITE_BAD_SHAPE, "gemm_rmsnorm: null pointer");
  if (!r && h_out) return fail(FERRITE_BAD_SHAPE, "gemm_rmsnorm: h_out needs a residual");
  if (ldx < k || ldx % 8 || ldc < n) return fail(FERRITE_BAD_SHAPE, "gemm_rmsnorm: leading dimension too small or not a multiple of 8");
  auto misaligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) != 0; };
  if (misaligned(x) || (r && misaligned(r)) || (h_out && misaligned(h_out)) || misaligned(w_norm))
    return fail(FERRITE_BAD_ALIGNMENT, "gemm_rmsnorm: x, r, h_out and w_norm must be 16-byte aligned");
  if (!(eps >= 0.f) || eps > 1.f) return fail(FERRITE_BAD_SHAPE, "gemm_rmsnorm: eps outside [0, 1]");
  if (h_out) {  // h_out is written while every CTA still reads x and r
    const uintptr_t span = (uintptr_t)(((m - 1) * ldx + k) * 2);
    auto overlaps = [&](const void* p) {
      const uintptr_t a0 = reinterpret_cast<uintptr_t>(p), b0 = reinterpret_cast<uintptr_t>(h_out);
      return a0 < b0 + span && b0 < a0 + span;
    };
    if (overlaps(x) || overlaps(r)) return fail(FERRITE_BAD_SHAPE, "gemm_rmsnorm: h_out overlaps x or r");
  }
  if (!skinny_kn_ok(b, m, n, k, ldb, 0, trans_b))
    return fail(FERRITE_UNSUPPORTED_DTYPE, "gemm_rmsnorm: B must be 16-byte aligned with ldb a multiple of 8 (and n a "
                                           "multiple of 8 when stored [K][N]), K within shared memory");
  cudaStream_t s = (cudaStream_t)stream;
  const KnNorm nrm{r, w_norm, h_out, eps};
  if (epilogue == kEpiGelu)
    return launch_skinny_kn<__nv_bfloat16, __nv_bfloat16, kEpiGelu, true>(s, x, b, c, m, n, k, ldx, ldb, ldc, 0, aux, ld_aux, nrm);
  if (ab_dtype == FERRITE_BF16) {
    if (c_dtype == FERRITE_F32)
      return launch_skinny_kn<__nv_bfloat16, float, kEpiNone, true>(s, x, b, c, m, n, k, ldx, ldb, ldc, trans_b, nullptr, 0, nrm);
    return launch_skinny_kn<__nv_bfloat16, __nv_bfloat16, kEpiNone, true>(s, x, b, c, m, n, k, ldx, ldb, ldc, trans_b, nullptr, 0, nrm);
  }
  if (c_dtype == FERRITE_F32)
    return launch_skinny_kn<__half, float, kEpiNone, true>(s, x, b, c, m, n, k, ldx, ldb, ldc, trans_b, nullptr, 0, nrm);
  return launch_skinny_kn<__half, __half, kEpiNone, true>(s, x, b, c, m, n, k, ldx, ldb, ldc, trans_b, nullptr, 0, nrm);
}

extern "C" int ferrite_gemm_epilogue(void* stream, const void* a, const void* b, void* c,
                                     int64_t m, int64_t n, int64_t k, int64_t lda, int64_t ldb,
                                     int64_t ldc, int trans_a, int trans_b, int epilogue,
                                     void* aux, int64_t ld_aux) {
  if (int rc = injected_fault("gemm")) return rc;
  if (epilogue != kEpiGelu && epilogue != kEpiGeluBwd)
    return fail(FERRITE_BAD_SHAPE, "gemm_epilogue: unknown epilogue %d", epilogue);
  if (m < 0 || n < 0 || k < 0) return fail(FERRITE_BAD_SHAPE, "gemm_epilogue: negative size");
  if (ld_aux < std::max<int64_t>(1, n) || ldc < std::max<int64_t>(1, n))
    return fail(FERRITE_BAD_SHAPE, "gemm_epilogue: leading dimension too small");
  if (m == 0 || n == 0) return FERRITE_OK;
  if (!a || !b || !c || !aux) return fail(FERRITE_BAD_SHAPE, "gemm_epilogue: null pointer");
  // decode-sized up-projections (at most 16 rows, W stored [K][N]): the skinny kernel
  if (epilogue == kEpiGelu && !trans_b && k > 0 && !tc_eligible(a, b, m, n, k, lda, ldb, trans_a, trans_b) &&
      skinny_kn_ok(b, m, n, k, ldb, trans_a, trans_b))
    return launch_skinny_kn<__nv_bfloat16, __nv_bfloat16, kEpiGelu>((cudaStream_t)stream, a, b, c, m, n, k, lda, ldb,
                                                                     ldc, 0, aux, ld_aux);
  if (k == 0 || !tc_eligible(a, b, m, n, k, lda, ldb, trans_a, trans_b))
    return fail(FERRITE_UNSUPPORTED_DTYPE,
                "gemm_epilogue: needs the tensor-core path (16-byte aligned operands and strides, "
                "m, n >= 128, k >= 64) or, for the GELU epilogue, the skinny path (m <= 16, B stored "
                "[K][N] 16-byte aligned, n and ldb multiples of 8)");
  return run_tc<true, __nv_bfloat16>((cudaStream_t)stream, a, b, c, m, n, k, lda, ldb, ldc, trans_a,
                                     trans_b, nullptr, 0, epilogue, aux, ld_aux);
}

extern "C" int ferrite_gemm_ws(void* stream, const void* a, const void* b, void* c, int64_t m,
                               int64_t n, int64_t k, int64_t lda, int64_t ldb, int64_t ldc,
                               int trans_a, int trans_b, int ab_dtype, int c_dtype,
                               void* workspace, size_t workspace_bytes) {
  if (int rc = injected_fault("gemm")) return rc;
  if (m < 0 || n < 0 || k < 0)
    return fail(FERRITE_BAD_SHAPE, "gemm: negative size m=%lld n=%lld k=%lld", (long long)m,
                (long long)n, (long long)k);
  const int64_t a_rows = trans_a ? k : m, a_cols = trans_a ? m : k;
  const int64_t b_rows = trans_b ? n : k, b_cols = trans_b ? k : n;
  if (lda < std::max<int64_t>(1, a_cols) || ldb < std::max<int64_t>(1, b_cols) ||
      ldc < std::max<int64_t>(1, n))
    return fail(FERRITE_BAD_SHAPE, "gemm: leading dimension too small (lda=%lld ldb=%lld ldc=%lld)",
                (long long)lda, (long long)ldb, (long long)ldc);
  (void)a_rows;
  (void)b_rows;
  if (ab_dtype != FERRITE_F32 && ab_dtype != FERRITE_BF16 && ab_dtype != FERRITE_F16)
    return fail(FERRITE_UNSUPPORTED_DTYPE, "gemm: operand dtype %d", ab_dtype);
  if (c_dtype != FERRITE_F32 && c_dtype != FERRITE_BF16 && c_dtype != FERRITE_F16)
    return fail(FERRITE_UNSUPPORTED_DTYPE, "gemm: output dtype %d", c_dtype);
  if (m == 0 || n == 0) return FERRITE_OK;
  if (!a || !b || !c) return fail(FERRITE_BAD_SHAPE, "gemm: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  if (k == 0) {
    // C = 0 (row by row to honour ldc)
    const size_t es = c_dtype == FERRITE_F32 ? 4 : 2;
    cudaError_t e = cudaMemset2DAsync(c, ldc * es, 0, n * es, m, s);
    return e == cudaSuccess ? FERRITE_OK : fail(FERRITE_LAUNCH_FAILED, "gemm: memset");
  }

  if (ab_dtype != FERRITE_F32 && tc_eligible(a, b, m, n, k, lda, ldb, trans_a, trans_b)) {
    const bool bf = ab_dtype == FERRITE_BF16;
    if (bf) {
      if (c_dtype == FERRITE_BF16) return run_tc<true, __nv_bfloat16>(s, a, b, c, m, n, k, lda, ldb, ldc, trans_a, trans_b, workspace, workspace_bytes);
      if (c_dtype == FERRITE_F32) return run_tc<true, float>(s, a, b, c, m, n, k, lda, ldb, ldc, trans_a, trans_b, workspace, workspace_bytes);
      return run_tc<true, __half>(s, a, b, c, m, n, k, lda, ldb, ldc, trans_a, trans_b, workspace, workspace_bytes);
    }
    if (c_dtype == FERRITE_BF16) return run_tc<false, __nv_bfloat16>(s, a, b, c, m, n, k, lda, ldb, ldc, trans_a, trans_b, workspace, workspace_bytes);
    if (c_dtype == FERRITE_F32) return run_tc<false, float>(s, a, b, c, m, n, k, lda, ldb, ldc, trans_a, trans_b, workspace, workspace_bytes);
    return run_tc<false, __half>(s, a, b, c, m, n, k, lda, ldb, ldc, trans_a, trans_b, workspace, workspace_bytes);
  }
  if (ab_dtype != FERRITE_F32 && skinny_kn_ok(b, m, n, k, ldb, trans_a, trans_b)) {
#define SKINNY_KN(TA, TC) launch_skinny_kn<TA, TC>(s, a, b, c, m, n, k, lda, ldb, ldc, trans_b)
    if (ab_dtype == FERRITE_BF16) {
      if (c_dtype == FERRITE_F32) return SKINNY_KN(__nv_bfloat16, float);
      if (c_dtype == FERRITE_BF16) return SKINNY_KN(__nv_bfloat16, __nv_bfloat16);
      return SKINNY_KN(__nv_bfloat16, __half);
    }
    if (c_dtype == FERRITE_F32) return SKINNY_KN(__half, float);
    if (c_dtype == FERRITE_BF16) return SKINNY_KN(__half, __nv_bfloat16);
    return SKINNY_KN(__half, __half);
#undef SKINNY_KN
  }
#define SIMT(TA, TC) launch_simt<TA, TC>(s, a, b, c, m, n, k, lda, ldb, ldc, trans_a, trans_b)
  if (ab_dtype == FERRITE_F32) {
    if (c_dtype == FERRITE_F32) return SIMT(float, float);
    if (c_dtype == FERRITE_BF16) return SIMT(float, __nv_bfloat16);
    return SIMT(float, __half);
  }
  if (ab_dtype == FERRITE_BF16) {
    if (c_dtype == FERRITE_F32) return SIMT(__nv_bfloat16, float);
    if (c_dtype == FERRITE_BF16) return SIMT(__nv_bfloat16, __nv_bfloat16);
    return SIMT(__nv_bfloat16, __half);
  }
  if (c_dtype == FERRITE_F32) return SIMT(__half, float);
  if (c_dtype == FERRITE_BF16) return SIMT(__half, __nv_bfloat16);
  return SIMT(__half, __half);
#undef SIMT
}

// ---------------------------------------------------------------------------
// Bounded-wait check: the failure path every tcgen05 kernel here takes when an
// mbarrier wait runs out, exercised on purpose with a short limit.
// ---------------------------------------------------------------------------
namespace ferrite {
namespace gemm {

// One CTA of four warps, laid out like the tensor-core kernels: warp 1 holds a
// TMEM allocation; lane 0 of warp 1 (the "MMA issuer") waits on an mbarrier that
// nothing ever arrives on, for at most `limit_ns`; lane 0 of warps 0, 2 and 3
// wait on a second such barrier and leave through the CTA's abort flag.  The
// expired wait records FERRITE_DEVICE_TIMEOUT in the status word.  Teardown is
// the kernels' own: __syncthreads, then the allocating warp frees TMEM.
// out[0] = ns the issuer waited, out[1] = 1 if its wait reported a timeout,
// out[2] = number of waiters that left (4), out[3] = 1 once TMEM was freed.
__global__ void __launch_bounds__(128) wait_probe_kernel(uint64_t limit_ns,
                                                         unsigned long long* out) {
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  __shared__ int left;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  volatile int* abort = &abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    abort_flag = 0;
    left = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, 32);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  if (lane == 0) {
    if (warp == 1) {
      const uint64_t t0 = globaltimer_ns();
      const bool ok = mbar_wait_ns(&bars[0], 0, abort, 90, limit_ns);
      out[0] = globaltimer_ns() - t0;
      out[1] = ok ? 0ull : 1ull;
    } else {
      // a bound 4x longer, so these leave through the abort flag the issuer raises
      (void)mbar_wait_ns(&bars[1], 0, abort, 91, 4 * limit_ns);
    }
    atomicAdd(&left, 1);
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 32);
    __syncwarp();
    if (lane == 0) {
      out[2] = (unsigned long long)left;
      out[3] = 1ull;
    }
  }
}

}  // namespace gemm
}  // namespace ferrite

extern "C" FERRITE_API int ferrite_wait_probe(void* stream, uint64_t limit_ns, void* out) {
  using namespace ferrite;
  if (limit_ns == 0 || limit_ns > kWaitLimitNs)
    return fail(FERRITE_BAD_SHAPE, "wait_probe: limit %llu ns outside (0, %llu]",
                (unsigned long long)limit_ns, (unsigned long long)kWaitLimitNs);
  if (!out || (reinterpret_cast<uintptr_t>(out) & 7u))
    return fail(FERRITE_BAD_ALIGNMENT, "wait_probe: out must be an 8-byte aligned device pointer");
  gemm::wait_probe_kernel<<<1, 128, 0, (cudaStream_t)stream>>>(limit_ns, (unsigned long long*)out);
  return check_launch("wait_probe");
}
