// csn_scan8.cu -- D = 8 (Cl(6,0) ~ M_8(R)) fused rotor scan, staged kernels.
//
// Same reduce -> carry -> apply algorithm as csn_scan.cu (one thread per (sequence,
// chunk)), specialised for the LM hot path:
//  * every step's inputs (generators, S or dX, X_{t-1}, gamma, dt) are staged with
//    cp.async into a private shared-memory slot of the thread; each slot is refilled
//    for the next step right after its last read in the current step, so the copy
//    overlaps (at least) the rest of the step's arithmetic;
//  * slot strides are 4 or 28 (mod 32) words, so the 8 lanes of a quarter warp hit 8
//    different bank groups in every 128-bit access pattern used here (own-slot rows and
//    the 4-lanes-per-row cooperative copies);
//  * rows that whole warps move (S, dX, X_{t-1}, X, dS, generators in the apply passes)
//    are copied cooperatively, 64 contiguous bytes of 8 rows per warp instruction;
//  * matrices that would not fit in the 255-register budget next to the live state
//    (the running product P in the reduce passes, M in the backward apply pass) live in
//    the slot too, and products with them are written as row-broadcast outer products
//    (one 128-bit load of a row feeds 32 FMAs), so they cost no register spills;
//  * the 8 x 8 products run on packed fp32 (fma.rn.f32x2: two adjacent entries of a row or
//    column per instruction, the other factor broadcast), which halves the FP32
//    instructions of the products without changing a single rounding: within a chunk the
//    forward state, the chunk aggregates and the gradient carry are bit-identical to the
//    scalar form.
// Chunks and the order of every accumulation in the forward pass match the generic kernels.
#include "csn_common.cuh"
#include "csn_internal.h"
#include "csn_scan_args.cuh"
#include "csn_carry.cuh"

namespace csn {
namespace s8 {

constexpr int DD = 64;
constexpr int K = 28;  // so(8) generators, reference triu layout
constexpr int THREADS = 128;

// slot layouts (floats)
struct FwdSlot {  // reduce / apply forward
  static constexpr int G = 0, S = 28, GAM = 92, DT = 93, P = 96, STRIDE = 164;
};
struct BwdRedSlot {  // backward reduce
  static constexpr int G = 0, DX = 28, GAM = 92, DT = 93, P = 96, STRIDE = 164;
};
struct BwdAppSlot {  // backward apply: M/S share a buffer
  static constexpr int MS = 0, XP = 64, DX = 128, G = 192, STRIDE = 220;
};
static_assert(FwdSlot::STRIDE % 32 == 4 && BwdRedSlot::STRIDE % 32 == 4, "bank spread");
static_assert(BwdAppSlot::STRIDE % 32 == 28, "bank spread");

extern __shared__ __align__(16) float s8_smem[];

__device__ __forceinline__ void lds_row(float (&r)[8], const float* p) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  const float4 b = *reinterpret_cast<const float4*>(p + 4);
  r[0] = a.x; r[1] = a.y; r[2] = a.z; r[3] = a.w; r[4] = b.x; r[5] = b.y; r[6] = b.z; r[7] = b.w;
}
__device__ __forceinline__ void sts_row(float* p, const float (&r)[8]) {
  *reinterpret_cast<float4*>(p) = make_float4(r[0], r[1], r[2], r[3]);
  *reinterpret_cast<float4*>(p + 4) = make_float4(r[4], r[5], r[6], r[7]);
}
__device__ __forceinline__ void lds_row2(uint64_t (&r)[4], const float* p) {
  const ulonglong2 a = *reinterpret_cast<const ulonglong2*>(p);
  const ulonglong2 b = *reinterpret_cast<const ulonglong2*>(p + 4);
  r[0] = a.x; r[1] = a.y; r[2] = b.x; r[3] = b.y;
}
__device__ __forceinline__ void sts_row2(float* p, const uint64_t (&r)[4]) {
  *reinterpret_cast<ulonglong2*>(p) = make_ulonglong2(r[0], r[1]);
  *reinterpret_cast<ulonglong2*>(p + 4) = make_ulonglong2(r[2], r[3]);
}
__device__ __forceinline__ float f2lo(uint64_t v) { return f2unpack(v).x; }
__device__ __forceinline__ float f2hi(uint64_t v) { return f2unpack(v).y; }

// ------------------------------------------------------ packed 8 x 8 products
// The products below are the scalar lmul / rmulT / lmulT / rmul of csn_common.cuh with two
// adjacent outputs per fma.rn.f32x2: every output entry sees the same fmaf chain in the same
// order (k = 0 first, as a product, then accumulated), so the results are bit-identical to
// the scalar forms, with half the FP32 instructions.  The paired operand is a pair of
// adjacent entries of M (down a column for lmul8p / rmulT8p, along a row for lmulT8p /
// rmul8p), the other factor one entry broadcast to both halves.

// X <- M X, columns 2q and 2q+1 at a time (in place: they depend only on themselves)
__device__ __forceinline__ void lmul8p(const Mat<8>& M, Mat<8>& X) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint64_t z0[4], z1[4];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint64_t s0 = f2splat(X.a[k][2 * q]), s1 = f2splat(X.a[k][2 * q + 1]);
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const uint64_t m = f2pack(M.a[2 * p][k], M.a[2 * p + 1][k]);
        z0[p] = k ? f2fma(m, s0, z0[p]) : f2mul(m, s0);
        z1[p] = k ? f2fma(m, s1, z1[p]) : f2mul(m, s1);
      }
    }
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      X.a[2 * p][2 * q] = f2lo(z0[p]);
      X.a[2 * p + 1][2 * q] = f2hi(z0[p]);
      X.a[2 * p][2 * q + 1] = f2lo(z1[p]);
      X.a[2 * p + 1][2 * q + 1] = f2hi(z1[p]);
    }
  }
}

// X <- X M^T, rows 2u and 2u+1 at a time
__device__ __forceinline__ void rmulT8p(Mat<8>& X, const Mat<8>& M) {
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    uint64_t y0[4], y1[4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint64_t s0 = f2splat(X.a[2 * u][j]), s1 = f2splat(X.a[2 * u + 1][j]);
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const uint64_t m = f2pack(M.a[2 * p][j], M.a[2 * p + 1][j]);
        y0[p] = j ? f2fma(s0, m, y0[p]) : f2mul(s0, m);
        y1[p] = j ? f2fma(s1, m, y1[p]) : f2mul(s1, m);
      }
    }
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      X.a[2 * u][2 * p] = f2lo(y0[p]);
      X.a[2 * u][2 * p + 1] = f2hi(y0[p]);
      X.a[2 * u + 1][2 * p] = f2lo(y1[p]);
      X.a[2 * u + 1][2 * p + 1] = f2hi(y1[p]);
    }
  }
}

// X <- M^T X, columns 2q and 2q+1 at a time
__device__ __forceinline__ void lmulT8p(const Mat<8>& M, Mat<8>& X) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint64_t z0[4], z1[4];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint64_t s0 = f2splat(X.a[k][2 * q]), s1 = f2splat(X.a[k][2 * q + 1]);
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const uint64_t m = f2pack(M.a[k][2 * p], M.a[k][2 * p + 1]);
        z0[p] = k ? f2fma(m, s0, z0[p]) : f2mul(m, s0);
        z1[p] = k ? f2fma(m, s1, z1[p]) : f2mul(m, s1);
      }
    }
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      X.a[2 * p][2 * q] = f2lo(z0[p]);
      X.a[2 * p + 1][2 * q] = f2hi(z0[p]);
      X.a[2 * p][2 * q + 1] = f2lo(z1[p]);
      X.a[2 * p + 1][2 * q + 1] = f2hi(z1[p]);
    }
  }
}

// X <- X M, rows 2u and 2u+1 at a time
__device__ __forceinline__ void rmul8p(Mat<8>& X, const Mat<8>& M) {
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    uint64_t y0[4], y1[4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint64_t s0 = f2splat(X.a[2 * u][j]), s1 = f2splat(X.a[2 * u + 1][j]);
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const uint64_t m = f2pack(M.a[j][2 * p], M.a[j][2 * p + 1]);
        y0[p] = j ? f2fma(s0, m, y0[p]) : f2mul(s0, m);
        y1[p] = j ? f2fma(s1, m, y1[p]) : f2mul(s1, m);
      }
    }
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      X.a[2 * u][2 * p] = f2lo(y0[p]);
      X.a[2 * u][2 * p + 1] = f2hi(y0[p]);
      X.a[2 * u + 1][2 * p] = f2lo(y1[p]);
      X.a[2 * u + 1][2 * p + 1] = f2hi(y1[p]);
    }
  }
}

// X += c R for 8 rows R read from shared memory (row stride 8), pairs along the rows
__device__ __forceinline__ void add_rows8p(Mat<8>& X, const float* rows, float c) {
  const uint64_t c2 = f2splat(c);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    uint64_t r2[4];
    lds_row2(r2, rows + 8 * i);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint64_t x = f2fma(c2, r2[q], f2pack(X.a[i][2 * q], X.a[i][2 * q + 1]));
      X.a[i][2 * q] = f2lo(x);
      X.a[i][2 * q + 1] = f2hi(x);
    }
  }
}

// ------------------------------------------------- warp-cooperative row transfers
// A lane's per-step rows (S, dX, X_{t-1}, X, dS: 64 floats = 256 B; generators 28 floats)
// are contiguous in memory but far from its neighbours' rows.  Instead of each lane moving
// its own row 16 B at a time (every warp instruction then touches 32 rows), 4 lanes move
// one row together: one warp instruction copies 64 contiguous bytes of each of 8 rows, and
// a lane issues RF / 16 such copies per row, for 4 groups of 8 rows.  The owner's row base
// comes from a shuffle once per row.  Rows p and p + 4 of a group share each 8-lane phase
// of a 128-bit shared-memory access: with slot strides of 41 or 55 (mod 8) 16-byte units
// their 4 + 4 vectors fall in 8 different bank groups.
struct LaneRows {
  int64_t first;  // element index (b*T + t)*N + n of the lane's first step (forward order)
  int len;        // steps in the lane's chunk (0 for lanes past the end of the grid)
  int t0;         // time index of the first step
};
constexpr unsigned FULL = 0xffffffffu;

// Row of lane r at `step` (reverse order counts from the chunk's last step), shifted by
// `back` rows (1 = the previous time step).  Returns -1 when that time is before 0.
template <bool REVERSE>
__device__ __forceinline__ int64_t lane_row(int64_t first, int len, int t0, int step, int back,
                                            int64_t row_step) {
  const int k = REVERSE ? (len - 1 - step) : step;
  if (t0 + k - back < 0) return -1;
  return first + (int64_t)(k - back) * row_step;
}

// row handled by this lane inside an 8-row group
__device__ __forceinline__ int coop_row_in_group(int lane) { return ((lane >> 2) & 1) * 4 + (lane >> 3); }

// g -> smem, RF floats per row (RF % 4 == 0).
template <int RF, bool REVERSE>
__device__ __forceinline__ void coop_load_rows(float* warp_slots, int stride, int off,
                                               const float* __restrict__ g, const LaneRows& me,
                                               int step, int64_t row_step, int back = 0) {
  constexpr int RV = RF / 4, SUB = (RV + 3) / 4;
  const int lane = threadIdx.x & 31, c = lane & 3, rg = coop_row_in_group(lane);
#pragma unroll
  for (int v = 0; v < 4; ++v) {
    const int r = 8 * v + rg;
    const int64_t first = __shfl_sync(FULL, me.first, r);
    const int len = __shfl_sync(FULL, me.len, r);
    const int t0 = __shfl_sync(FULL, me.t0, r);
    if (step < len) {
      const int64_t row = lane_row<REVERSE>(first, len, t0, step, back, row_step);
      if (row >= 0) {
#pragma unroll
        for (int u = 0; u < SUB; ++u) {
          const int vec = 4 * u + c;
          if (vec < RV) cp_async16(warp_slots + r * stride + off + 4 * vec, g + row * RF + 4 * vec);
        }
      }
    }
  }
}

// smem -> g, each row scaled by its owner's `scale`.
template <int RF, bool REVERSE>
__device__ __forceinline__ void coop_store_rows(const float* warp_slots, int stride, int off,
                                                float* __restrict__ g, const LaneRows& me,
                                                int step, int64_t row_step, float scale) {
  constexpr int RV = RF / 4, SUB = (RV + 3) / 4;
  const int lane = threadIdx.x & 31, c = lane & 3, rg = coop_row_in_group(lane);
#pragma unroll
  for (int v = 0; v < 4; ++v) {
    const int r = 8 * v + rg;
    const int64_t first = __shfl_sync(FULL, me.first, r);
    const int len = __shfl_sync(FULL, me.len, r);
    const int t0 = __shfl_sync(FULL, me.t0, r);
    const float sc = __shfl_sync(FULL, scale, r);
    if (step < len) {
      const int64_t row = lane_row<REVERSE>(first, len, t0, step, 0, row_step);
#pragma unroll
      for (int u = 0; u < SUB; ++u) {
        const int vec = 4 * u + c;
        if (vec < RV) {
          float4 f = *reinterpret_cast<const float4*>(warp_slots + r * stride + off + 4 * vec);
          f.x *= sc; f.y *= sc; f.z *= sc; f.w *= sc;
          __stcs(reinterpret_cast<float4*>(g + row * RF + 4 * vec), f);
        }
      }
    }
  }
}

// M = sa (2 (I - Omega)^{-1} - I) from the staged generators.
template <bool DAMPED>
__device__ __forceinline__ void cayley_from_slot(const float* gslot, float dtv, float gam,
                                                 Mat<8>& M, float& alpha, float& sa) {
  float g[K];
#pragma unroll
  for (int v = 0; v < K / 4; ++v) {
    const float4 f = *reinterpret_cast<const float4*>(gslot + 4 * v);
    g[4 * v] = f.x; g[4 * v + 1] = f.y; g[4 * v + 2] = f.z; g[4 * v + 3] = f.w;
  }
  build_neg_omega<8, BASIS_TRIU, K>(M, g, 0.5f * dtv);
  gj_inverse_dev(M);  // (I - Omega)^{-1} - I
  if constexpr (DAMPED) {
    alpha = 1.0f / (1.0f + expf(gam * dtv));
    sa = sqrtf(alpha);
  } else {
    alpha = 1.0f;
    sa = 1.0f;
  }
  rotor_from_dev(M, sa);
}

__device__ __forceinline__ void thread_coords(const ScanArgs& a, int64_t tid, int64_t& b, int64_t& n,
                                              int64_t& j) {
  n = tid % a.N;
  j = (tid / a.N) % a.nchunks;
  b = tid / (a.N * a.nchunks);
}

// ------------------------------------------------------------------ forward
// REDUCE = true: chunk aggregate (P, c) with zero carry.  REDUCE = false: rescan from
// the chunk's carry and write X.  The step loop is warp-uniform (it runs to the longest
// chunk in the warp) because the S loads and X stores are warp-cooperative.
template <bool REDUCE, bool DAMPED, bool TWO>
__global__ void __launch_bounds__(THREADS, 2) fwd8_kernel(ScanArgs a) {
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t total = a.B * a.N * a.nchunks;
  const bool active = tid < total;
  int64_t b = 0, n = 0, j = 0;
  if (active) thread_coords(a, tid, b, n, j);
  const int64_t s = b * a.N + n;
  const int64_t t0 = j * a.chunk, t1 = active ? min(a.T, t0 + a.chunk) : t0;
  LaneRows me{(b * a.T + t0) * a.N + n, (int)(t1 - t0), (int)t0};
  const int nsteps = __reduce_max_sync(FULL, me.len);
  if (nsteps == 0) return;  // whole warp idle
  float* warp_slots = s8_smem + (threadIdx.x & ~31) * FwdSlot::STRIDE;
  float* slot = s8_smem + threadIdx.x * FwdSlot::STRIDE;

  auto issue_a = [&](int st) {  // generators, gamma, dt of step st (own lane)
    if (st < me.len) {
      const int64_t t = t0 + st;
      const int64_t e = (b * a.T + t) * a.N + n;
      cp_async_floats<K>(slot + FwdSlot::G, a.gens + e * K);
      if (DAMPED) cp_async4(slot + FwdSlot::GAM, a.gamma + e);
      cp_async4(slot + FwdSlot::DT, a.dt + dt_index(a, b, t, n));
    }
  };

  // S of step st: the apply pass loads it warp-cooperatively (coalesced); the reduce pass,
  // which is arithmetic-bound, lets each lane copy its own row (no shuffles)
  auto issue_s = [&](int st) {
    if constexpr (REDUCE) {
      if (st < me.len) {
        const int64_t e = (b * a.T + t0 + st) * a.N + n;
        cp_async_floats<DD>(slot + FwdSlot::S, a.S + e * DD);
      }
    } else {
      coop_load_rows<DD, false>(warp_slots, FwdSlot::STRIDE, FwdSlot::S, a.S, me, st, a.N);
    }
  };
  issue_a(0);
  cp_async_commit();
  issue_s(0);
  cp_async_commit();

  Mat<8> X, M;
  if constexpr (REDUCE) {
    mat_zero(X);
#pragma unroll
    for (int i = 0; i < 8; ++i) {  // P^T = I, stored transposed: row j of P^T = column j of P
      float r[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) r[c] = (i == c) ? 1.0f : 0.0f;
      sts_row(slot + FwdSlot::P + 8 * i, r);
    }
  } else {
    if (!active) mat_zero(X);
    else if (a.nchunks > 1) load_mat(X, a.carry + (s * a.nchunks + j) * DD);
    else if (a.h0) load_mat(X, a.h0 + s * DD);
    else mat_zero(X);
  }

  for (int st = 0; st < nsteps; ++st) {
    const bool live = st < me.len;
    cp_async_wait<1>();  // own generators / gamma / dt of this step
    float alpha = 1.0f, sa = 1.0f;
    if (live) {
      const float dtv = slot[FwdSlot::DT];
      const float gam = DAMPED ? slot[FwdSlot::GAM] : 0.0f;
      cayley_from_slot<DAMPED>(slot + FwdSlot::G, dtv, gam, M, alpha, sa);
    }
    issue_a(st + 1);
    cp_async_commit();
    if (live) {
      lmul8p(M, X);
      if constexpr (TWO) rmulT8p(X, M);
    }
    cp_async_wait<1>();  // S rows of this step
    if constexpr (!REDUCE) __syncwarp();  // rows were copied by other lanes
    const float cs = DAMPED ? (1.0f - alpha) : 1.0f;
    if (live) {
      if constexpr (TWO) {
        add_rows8p(X, slot + FwdSlot::S, cs);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float r[8];
          lds_row(r, slot + FwdSlot::S + 8 * i);
#pragma unroll
          for (int c = 0; c < 8; ++c) X.a[i][c] = fmaf(cs, r[c], X.a[i][c]);
        }
      }
    }
    if constexpr (REDUCE) {
      issue_s(st + 1);
      cp_async_commit();
      if (live) {
        // P <- M P; column j of the new P = M * (column j of P) = M * (row j of P^T)
        // (jj only addresses shared memory: rolled, 9 % faster than unrolled)
#pragma unroll 1
        for (int jj = 0; jj < 8; ++jj) {
          float v[8];
          uint64_t o2[4];
          lds_row(v, slot + FwdSlot::P + 8 * jj);
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const uint64_t sv = f2splat(v[k]);
#pragma unroll
            for (int p = 0; p < 4; ++p) {
              const uint64_t m = f2pack(M.a[2 * p][k], M.a[2 * p + 1][k]);
              o2[p] = k ? f2fma(m, sv, o2[p]) : f2mul(m, sv);
            }
          }
          sts_row2(slot + FwdSlot::P + 8 * jj, o2);
        }
      }
    } else {
      // X goes out through the S buffer: own row into the slot, then a coalesced store
      if (live) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float r[8];
#pragma unroll
          for (int c = 0; c < 8; ++c) r[c] = X.a[i][c];
          sts_row(slot + FwdSlot::S + 8 * i, r);
        }
      }
      __syncwarp();
      coop_store_rows<DD, false>(warp_slots, FwdSlot::STRIDE, FwdSlot::S, a.out, me, st, a.N, 1.0f);
      __syncwarp();  // the S buffer is free again
      issue_s(st + 1);
      cp_async_commit();
    }
  }
  cp_async_wait<0>();
  if (!active) return;
  if constexpr (REDUCE) {
    store_mat(a.aggC + (s * a.nchunks + j) * DD, X);
    Mat<8> P;
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) {
      float v[8];
      lds_row(v, slot + FwdSlot::P + 8 * jj);
#pragma unroll
      for (int i = 0; i < 8; ++i) P.a[i][jj] = v[i];
    }
    store_mat(a.aggP + (s * a.nchunks + j) * DD, P);
  }
}

// --------------------------------------------------------------- backward reduce
// g <- 0; for t = end .. start: G = dX_t + g; g = M^T G M (one-sided M^T G); P <- P M
template <bool DAMPED, bool TWO>
__global__ void __launch_bounds__(THREADS, 2) bwd8_reduce_kernel(ScanArgs a) {
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (tid >= a.B * a.N * a.nchunks) return;
  int64_t b, n, j;
  thread_coords(a, tid, b, n, j);
  if (j == 0 && !a.agg_mode) return;
  const int64_t s = b * a.N + n;
  const int64_t t0 = j * a.chunk, t1 = min(a.T, t0 + a.chunk);
  float* slot = s8_smem + threadIdx.x * BwdRedSlot::STRIDE;

  auto issue_a = [&](int64_t t) {
    const int64_t e = (b * a.T + t) * a.N + n;
    cp_async_floats<K>(slot + BwdRedSlot::G, a.gens + e * K);
    if (DAMPED) cp_async4(slot + BwdRedSlot::GAM, a.gamma + e);
    cp_async4(slot + BwdRedSlot::DT, a.dt + dt_index(a, b, t, n));
  };
  auto issue_b = [&](int64_t t) {
    const int64_t e = (b * a.T + t) * a.N + n;
    cp_async_floats<DD>(slot + BwdRedSlot::DX, a.dX + e * DD);
  };
  issue_a(t1 - 1);
  cp_async_commit();
  issue_b(t1 - 1);
  cp_async_commit();
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float r[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) r[c] = (i == c) ? 1.0f : 0.0f;
    sts_row(slot + BwdRedSlot::P + 8 * i, r);
  }
  Mat<8> g, M;
  mat_zero(g);
  for (int64_t t = t1 - 1; t >= t0; --t) {
    cp_async_wait<1>();
    const float dtv = slot[BwdRedSlot::DT];
    const float gam = DAMPED ? slot[BwdRedSlot::GAM] : 0.0f;
    float alpha, sa;
    cayley_from_slot<DAMPED>(slot + BwdRedSlot::G, dtv, gam, M, alpha, sa);
    if (t - 1 >= t0) issue_a(t - 1);
    cp_async_commit();
    cp_async_wait<1>();
    if constexpr (TWO) {
      add_rows8p(g, slot + BwdRedSlot::DX, 1.0f);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float r[8];
        lds_row(r, slot + BwdRedSlot::DX + 8 * i);
#pragma unroll
        for (int c = 0; c < 8; ++c) g.a[i][c] += r[c];
      }
    }
    if (t - 1 >= t0) issue_b(t - 1);
    cp_async_commit();
    lmulT8p(M, g);
    if constexpr (TWO) rmul8p(g, M);
    // P <- P M, row by row in place (i only addresses shared memory: rolled)
    if (!a.reuse_P) {
#pragma unroll 1
      for (int i = 0; i < 8; ++i) {
        float v[8];
        uint64_t o2[4];
        lds_row(v, slot + BwdRedSlot::P + 8 * i);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint64_t sv = f2splat(v[k]);
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            const uint64_t m = f2pack(M.a[k][2 * p], M.a[k][2 * p + 1]);
            o2[p] = k ? f2fma(sv, m, o2[p]) : f2mul(sv, m);
          }
        }
        sts_row2(slot + BwdRedSlot::P + 8 * i, o2);
      }
    }
  }
  cp_async_wait<0>();
  store_mat(a.aggC + (s * a.nchunks + j) * DD, g);
  if (a.reuse_P) return;
  Mat<8> P;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float v[8];
    lds_row(v, slot + BwdRedSlot::P + 8 * i);
#pragma unroll
    for (int l = 0; l < 8; ++l) P.a[i][l] = v[l];
  }
  store_mat(a.aggP + (s * a.nchunks + j) * DD, P);
}

// ---------------------------------------------------------------- backward apply
// Per step t (reverse):  G = dX_t + H
//   dS_t = (1 - a) G,  dM = G M Xp^T + G^T M Xp  (one-sided: G Xp^T),  Xp = X_{t-1}
//   da = -<G, S> + <dM, M> / (2 a)
//   V = (M^T dM + sa dM) / 2,  dOm = V M^T / sa + V,  dg_k = <dOm, E_k> dt / 2
//   H <- M^T G M  (one-sided: M^T G)
// Slot: [M or S | Xp | dX or G | gens or dgens].  S_t is staged into the M buffer and
// read before M_t overwrites it; G is parked in the dX buffer right after it is formed;
// dgens leaves through the generator buffer.  Every row moves warp-cooperatively
// (coalesced), so the step loop is warp-uniform.  Group order per step: Xp, gens, S+dX.
template <bool DAMPED, bool TWO>
__global__ void __launch_bounds__(THREADS, 2) bwd8_apply_kernel(ScanArgs a) {
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t total = a.B * a.N * a.nchunks;
  const bool active = tid < total;
  int64_t b = 0, n = 0, j = 0;
  if (active) thread_coords(a, tid, b, n, j);
  const int64_t s = b * a.N + n;
  const int64_t t0 = j * a.chunk, t1 = active ? min(a.T, t0 + a.chunk) : t0;
  const LaneRows me{(b * a.T + t0) * a.N + n, (int)(t1 - t0), (int)t0};
  const int nsteps = __reduce_max_sync(FULL, me.len);
  if (nsteps == 0) return;
  constexpr int ST = BwdAppSlot::STRIDE;
  float* warp_slots = s8_smem + (threadIdx.x & ~31) * ST;
  float* slot = s8_smem + threadIdx.x * ST;
  float* sM = slot + BwdAppSlot::MS;
  float* sXp = slot + BwdAppSlot::XP;
  float* sDX = slot + BwdAppSlot::DX;
  float* sG = slot + BwdAppSlot::G;

  // step st of this lane is time t = t1 - 1 - st
  auto issue_xp = [&](int st) {  // X_{t-1}; rows before t = 0 come from h0 (or zeros) below
    coop_load_rows<DD, true>(warp_slots, ST, BwdAppSlot::XP, a.X, me, st, a.N, 1);
  };
  auto fix_xp = [&](int st) {  // own lane: X_{-1} = h0 or 0 when this step is t = 0
    if (st < me.len && t1 - 1 - st == 0) {
      if (a.h0) {
#pragma unroll
        for (int v = 0; v < 16; ++v)
          *reinterpret_cast<float4*>(sXp + 4 * v) = __ldg(reinterpret_cast<const float4*>(a.h0 + s * DD) + v);
      } else {
        float z[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
        for (int i = 0; i < 8; ++i) sts_row(sXp + 8 * i, z);
      }
    }
  };
  auto issue_gens = [&](int st) {
    coop_load_rows<K, true>(warp_slots, ST, BwdAppSlot::G, a.gens, me, st, a.N);
  };
  auto issue_sdx = [&](int st) {
    if (DAMPED) coop_load_rows<DD, true>(warp_slots, ST, BwdAppSlot::MS, a.S, me, st, a.N);
    coop_load_rows<DD, true>(warp_slots, ST, BwdAppSlot::DX, a.dX, me, st, a.N);
  };
  issue_xp(0);
  cp_async_commit();
  issue_gens(0);
  cp_async_commit();
  issue_sdx(0);
  cp_async_commit();
  fix_xp(0);
  float gam_n = 0.0f, dt_n = 0.0f;
  if (me.len > 0) {
    const int64_t e = (b * a.T + t1 - 1) * a.N + n;
    if (DAMPED) gam_n = __ldg(a.gamma + e);
    dt_n = __ldg(a.dt + dt_index(a, b, t1 - 1, n));
  }

  // packed state and gradients: entry pairs (c, c+1) of a row in one 64-bit register pair
  uint64_t H2[8][4];
  {
    Mat<8> H;
    if (active && a.nchunks > 1) load_mat(H, a.carry + (s * a.nchunks + j) * DD);
    else if (active && a.hT) load_mat(H, a.hT + s * DD);
    else mat_zero(H);
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int q = 0; q < 4; ++q) H2[i][q] = f2pack(H.a[i][2 * q], H.a[i][2 * q + 1]);
  }

  for (int st = 0; st < nsteps; ++st) {
    const bool live = st < me.len;
    const int64_t t = t1 - 1 - st;
    const int64_t e = (b * a.T + t) * a.N + n;
    const float dtv = dt_n, gam = gam_n;
    if (st + 1 < me.len) {  // scalars of the next step, a full step ahead
      const int64_t e1 = (b * a.T + t - 1) * a.N + n;
      if (DAMPED) gam_n = __ldg(a.gamma + e1);
      dt_n = __ldg(a.dt + dt_index(a, b, t - 1, n));
    }
    // ---- 1. Cayley in registers (Xp, gens landed; S, dX may still be in flight)
    cp_async_wait<1>();
    __syncwarp();
    Mat<8> Mr;
    float alpha = 1.0f, sa = 1.0f;
    if (live) cayley_from_slot<DAMPED>(sG, dtv, gam, Mr, alpha, sa);
    // ---- 2. G = H + dX;  <G, S>;  G parks in the dX buffer;  M into its buffer
    cp_async_wait<0>();
    __syncwarp();
    uint64_t gS2 = 0;
    const float cs = DAMPED ? (1.0f - alpha) : 1.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      uint64_t r2[4], s2[4];
      lds_row2(r2, sDX + 8 * i);
      if (DAMPED) lds_row2(s2, sM + 8 * i);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        H2[i][q] = f2add(H2[i][q], r2[q]);
        if (DAMPED) gS2 = f2fma(H2[i][q], s2[q], gS2);
      }
      sts_row2(sDX + 8 * i, H2[i]);
    }
    const float gS = f2sum(gS2);
#pragma unroll
    for (int i = 0; i < 8; ++i) sts_row(sM + 8 * i, Mr.a[i]);
    __syncwarp();
    coop_store_rows<DD, true>(warp_slots, ST, BwdAppSlot::DX, a.dC, me, st, a.N, cs);  // dS = (1-a) G
    // ---- 3. dM, with G read back from the dX buffer
    uint64_t dM2[8][4];
    if constexpr (TWO) {
      // dM = (G M) Xp^T + (G^T M) Xp.  First the G^T M part, which reads every column of G;
      // then G M by halves of rows: half h reads only rows 4h..4h+3 of G, so its rows of G M
      // replace them in the dX buffer, where the state update H = M^T (G M) reads them.
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        // keeps the scheduler from overlapping the two halves (which would hold both
        // halves' temporaries at once and spill)
        __syncwarp();
        uint64_t U2[4][4];
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
          for (int q = 0; q < 4; ++q) U2[r][q] = 0;
        // k only addresses shared memory here, so the loop stays rolled (smaller step body)
#pragma unroll 1
        for (int k = 0; k < 8; ++k) {  // U = (G^T)[rows] M
          uint64_t mr2[4];
          lds_row2(mr2, sM + 8 * k);
          const float4 gu4 = *reinterpret_cast<const float4*>(sDX + 8 * k + 4 * h);  // G[k][rows]
          const float guv[4] = {gu4.x, gu4.y, gu4.z, gu4.w};
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const uint64_t gg = f2splat(guv[r]);
#pragma unroll
            for (int q = 0; q < 4; ++q) U2[r][q] = f2fma(gg, mr2[q], U2[r][q]);
          }
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {  // dM[rows] = U Xp
          uint64_t xr2[4];
          lds_row2(xr2, sXp + 8 * k);
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const float2 up = f2unpack(U2[r][k >> 1]);
            const uint64_t uu = f2splat((k & 1) ? up.y : up.x);
#pragma unroll
            for (int q = 0; q < 4; ++q)
              dM2[4 * h + r][q] = (k == 0) ? f2mul(uu, xr2[q]) : f2fma(uu, xr2[q], dM2[4 * h + r][q]);
          }
        }
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        __syncwarp();
        uint64_t W2[4][4];
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
          for (int q = 0; q < 4; ++q) W2[r][q] = 0;
#pragma unroll 1
        for (int k = 0; k < 8; ++k) {  // W = G[rows] M
          uint64_t mr2[4];
          lds_row2(mr2, sM + 8 * k);
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const uint64_t gg = f2splat(sDX[8 * (4 * h + r) + k]);
#pragma unroll
            for (int q = 0; q < 4; ++q) W2[r][q] = f2fma(gg, mr2[q], W2[r][q]);
          }
        }
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {  // dM[rows][k] += W[rows] . Xp[k], k = 2kk, 2kk+1
          uint64_t xa[4], xb[4];
          lds_row2(xa, sXp + 16 * kk);
          lds_row2(xb, sXp + 16 * kk + 8);
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            uint64_t pa = f2mul(W2[r][0], xa[0]), pb = f2mul(W2[r][0], xb[0]);
#pragma unroll
            for (int q = 1; q < 4; ++q) {
              pa = f2fma(W2[r][q], xa[q], pa);
              pb = f2fma(W2[r][q], xb[q], pb);
            }
            dM2[4 * h + r][kk] = f2add(dM2[4 * h + r][kk], f2pack(f2sum(pa), f2sum(pb)));
          }
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) sts_row2(sDX + 8 * (4 * h + r), W2[r]);  // rows of G M over rows of G
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) {  // dM = G Xp^T, row i from row i of G
        float gr[8], d[8];
        lds_row(gr, sDX + 8 * i);
#pragma unroll
        for (int l = 0; l < 8; ++l) {
          float xr[8];
          lds_row(xr, sXp + 8 * l);
          float acc = 0.0f;
#pragma unroll
          for (int k = 0; k < 8; ++k) acc = fmaf(gr[k], xr[k], acc);
          d[l] = acc;
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) dM2[i][q] = f2pack(d[2 * q], d[2 * q + 1]);
      }
    }
    __syncwarp();  // every lane is done with its Xp
    issue_xp(st + 1);
    cp_async_commit();
    fix_xp(st + 1);
    // ---- 4. decay gradient
    float da = 0.0f;
    if constexpr (DAMPED) {
      uint64_t dmm2 = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        uint64_t mr2[4];
        lds_row2(mr2, sM + 8 * i);
#pragma unroll
        for (int q = 0; q < 4; ++q) dmm2 = f2fma(dM2[i][q], mr2[q], dmm2);
      }
      da = -gS + f2sum(dmm2) / (2.0f * alpha);
    }
    // ---- 5. generator gradient: V = (M^T dM + sa dM)/2, dOm = V M^T / sa + V
    float proj[K];
#pragma unroll
    for (int k = 0; k < K; ++k) proj[k] = 0.0f;
    {
      const float inv_sa = 1.0f / sa;
      const uint64_t sa2 = f2splat(sa), half2 = f2splat(0.5f);
#pragma unroll
      for (int h = 0; h < 2; ++h) {  // rows 4h .. 4h+3 of V and dOm
        __syncwarp();
        uint64_t V2[4][4];
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
          for (int q = 0; q < 4; ++q) V2[r][q] = f2mul(sa2, dM2[4 * h + r][q]);
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {  // V += (M^T dM)[rows]
          const float4 m4 = *reinterpret_cast<const float4*>(sM + 8 * jj + 4 * h);
          const float mv[4] = {m4.x, m4.y, m4.z, m4.w};
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const uint64_t mm = f2splat(mv[r]);
#pragma unroll
            for (int q = 0; q < 4; ++q) V2[r][q] = f2fma(mm, dM2[jj][q], V2[r][q]);
          }
        }
#pragma unroll
        for (int r = 0; r < 4; ++r)  // V /= 2 (exact)
#pragma unroll
          for (int q = 0; q < 4; ++q) V2[r][q] = f2mul(half2, V2[r][q]);
#pragma unroll
        for (int l = 0; l < 8; ++l) {  // dOm[rows][l] = (V M^T)[rows][l] / sa + V[rows][l]
          uint64_t mr2[4];
          lds_row2(mr2, sM + 8 * l);
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const int i = 4 * h + r;
            if (i == l) continue;
            uint64_t acc2 = f2mul(V2[r][0], mr2[0]);
#pragma unroll
            for (int q = 1; q < 4; ++q) acc2 = f2fma(V2[r][q], mr2[q], acc2);
            const float2 vp = f2unpack(V2[r][l >> 1]);
            const float dom = fmaf(f2sum(acc2), inv_sa, (l & 1) ? vp.y : vp.x);
            if (i < l) proj[i * (15 - i) / 2 + (l - i - 1)] += dom;
            else proj[l * (15 - l) / 2 + (i - l - 1)] -= dom;
          }
        }
      }
    }
    {
      const float hdt = 0.5f * dtv;
      float ddt = 0.0f;
#pragma unroll
      for (int v = 0; v < K / 4; ++v) {  // g_t is still in the generator buffer
        float4 f = *reinterpret_cast<const float4*>(sG + 4 * v);
        ddt = fmaf(proj[4 * v], 0.5f * f.x, ddt);
        ddt = fmaf(proj[4 * v + 1], 0.5f * f.y, ddt);
        ddt = fmaf(proj[4 * v + 2], 0.5f * f.z, ddt);
        ddt = fmaf(proj[4 * v + 3], 0.5f * f.w, ddt);
        f = make_float4(proj[4 * v] * hdt, proj[4 * v + 1] * hdt, proj[4 * v + 2] * hdt,
                        proj[4 * v + 3] * hdt);
        *reinterpret_cast<float4*>(sG + 4 * v) = f;  // dgens leave through the same buffer
      }
      if (live) {
        if constexpr (DAMPED) {
          const float dz = da * alpha * (1.0f - alpha);
          a.dgamma[e] = -dz * dtv;
          ddt = fmaf(-dz, gam, ddt);
        }
        a.ddt_part[e] = ddt;
      }
    }
    __syncwarp();
    coop_store_rows<K, true>(warp_slots, ST, BwdAppSlot::G, a.dgens, me, st, a.N, 1.0f);
    __syncwarp();
    issue_gens(st + 1);
    cp_async_commit();
    // ---- 6. H <- M^T (G M) (one-sided: M^T G): rows of G M (two-sided) or of G (one-sided)
    // are read back from the dX buffer
    {
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int q = 0; q < 4; ++q) H2[i][q] = 0;
#pragma unroll 1  // k only addresses shared memory (rolled, as above)
      for (int k = 0; k < 8; ++k) {
        float mr[8];
        uint64_t gr2[4];
        lds_row(mr, sM + 8 * k);
        lds_row2(gr2, sDX + 8 * k);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint64_t mm = f2splat(mr[i]);
#pragma unroll
          for (int q = 0; q < 4; ++q) H2[i][q] = f2fma(mm, gr2[q], H2[i][q]);
        }
      }
    }
    __syncwarp();  // M and G buffers are free
    issue_sdx(st + 1);
    cp_async_commit();
  }
  cp_async_wait<0>();
  if (active && j == 0 && a.dh0) {
    Mat<8> H;
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 p = f2unpack(H2[i][q]);
        H.a[i][2 * q] = p.x;
        H.a[i][2 * q + 1] = p.y;
      }
    store_mat(a.dh0 + s * DD, H);
  }
}

template <typename Kern>
void set_smem(Kern k, int bytes) {
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

unsigned nblk(int64_t n) { return (unsigned)((n + THREADS - 1) / THREADS); }

template <bool DAMPED, bool TWO>
int run8(const ScanArgs& a, bool bwd, cudaStream_t st) {
  const int64_t S = a.B * a.N;
  const int64_t total = S * a.nchunks;
  const int fwd_bytes = THREADS * FwdSlot::STRIDE * 4;
  const int red_bytes = THREADS * BwdRedSlot::STRIDE * 4;
  const int app_bytes = THREADS * BwdAppSlot::STRIDE * 4;
  if (a.agg_mode == 1) {
    if (total == 0) return CSN_OK;
    if (!bwd) {
      {
        KernelTimer kt("agg_fwd_reduce", st);
        set_smem(fwd8_kernel<true, DAMPED, TWO>, fwd_bytes);
        fwd8_kernel<true, DAMPED, TWO><<<nblk(total), THREADS, fwd_bytes, st>>>(a);
      }
      KernelTimer kt("agg_compose", st);
      launch_compose8_mma<TWO, false>(a, st);
    } else {
      {
        KernelTimer kt("agg_bwd_reduce", st);
        set_smem(bwd8_reduce_kernel<DAMPED, TWO>, red_bytes);
        bwd8_reduce_kernel<DAMPED, TWO><<<nblk(total), THREADS, red_bytes, st>>>(a);
      }
      KernelTimer kt("agg_compose", st);
      launch_compose8_mma<TWO, true>(a, st);
    }
    return check_launch("shard aggregate (D=8)");
  }
  if (!bwd) {
    if (total == 0) return CSN_OK;
    if (a.nchunks > 1) {
      if (a.agg_mode != 2) {
        KernelTimer kt("fwd_reduce", st);
        set_smem(fwd8_kernel<true, DAMPED, TWO>, fwd_bytes);
        fwd8_kernel<true, DAMPED, TWO><<<nblk(total), THREADS, fwd_bytes, st>>>(a);
      }
      KernelTimer kt("fwd_carry", st);
      launch_grouped_carry<8, TWO, false>(a, st);
    }
    KernelTimer kt("fwd_apply", st);
    set_smem(fwd8_kernel<false, DAMPED, TWO>, fwd_bytes);
    fwd8_kernel<false, DAMPED, TWO><<<nblk(total), THREADS, fwd_bytes, st>>>(a);
    return check_launch("rotor scan forward (D=8)");
  }
  if (total > 0) {
    if (a.nchunks > 1) {
      if (a.agg_mode != 2) {
        KernelTimer kt("bwd_reduce", st);
        set_smem(bwd8_reduce_kernel<DAMPED, TWO>, red_bytes);
        bwd8_reduce_kernel<DAMPED, TWO><<<nblk(total), THREADS, red_bytes, st>>>(a);
      }
      KernelTimer kt("bwd_carry", st);
      launch_grouped_carry<8, TWO, true>(a, st);
    }
    KernelTimer kt("bwd_apply", st);
    set_smem(bwd8_apply_kernel<DAMPED, TWO>, app_bytes);
    bwd8_apply_kernel<DAMPED, TWO><<<nblk(total), THREADS, app_bytes, st>>>(a);
  }
  if (a.B * a.T > 0) {
    const int64_t BT = a.B * a.T;
    KernelTimer kt("reduce_channels", st);
    const int64_t H = dt_heads(a);
    reduce_channels_kernel<<<(unsigned)((BT * H + 255) / 256), 256, 0, st>>>(a.ddt_part, a.ddt, BT * H,
                                                                            a.N / H);
  }
  return check_launch("rotor scan backward (D=8)");
}

// ------------------------------------------------------------- single step (generation)
// One step X <- M X M^T + (1 - alpha) S (one-sided: M X) of B x N independent states,
// row-parallel: eight lanes per state, lane r owns row r of A = I - Omega, of M and of X.
// The Gauss-Jordan pivot row is broadcast within the 8-lane group by shuffles; the rows of
// X and M that the products need go through shared memory.  The arithmetic per entry is
// the same sequence as the sequential scan (build_neg_omega, gj_inverse_dev, lmul, rmulT),
// so a step equals the scan's step.
constexpr int STEP_THREADS = 128;

// CHAINED: launched with programmatic stream serialization after another step: the kernel
// lets the next step launch at once, builds its rotor (which reads only this step's
// generators, dt, gamma and S) while the previous step is still running, and reads the state
// only after griddepcontrol.wait, i.e. after the previous grid has completed and its writes
// are visible.  The inputs must therefore not be written by the kernel launched before it.
template <bool DAMPED, bool TWO, bool CHAINED>
__global__ void __launch_bounds__(STEP_THREADS) step8_kernel(const float* __restrict__ gens,
                                                             const float* __restrict__ dt,
                                                             const float* __restrict__ gamma,
                                                             const float* __restrict__ S,
                                                             float* h, int64_t B, int64_t N) {
  if constexpr (CHAINED) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __shared__ __align__(16) float sX[STEP_THREADS / 8][DD];
  __shared__ __align__(16) float sM[STEP_THREADS / 8][DD];
  const int r = threadIdx.x & 7;
  const int grp = threadIdx.x >> 3;
  const int64_t e = blockIdx.x * (int64_t)(STEP_THREADS / 8) + grp;  // state index b * N + n
  const bool active = e < B * N;  // uniform over the 8-lane group
  const int64_t b = active ? e / N : 0;

  // row r of A = I - (dt / 2) Omega; generator k of the pair (u, v), u < v, row-major
  // the state and S rows do not depend on the rotor: issue their loads first so that their
  // latency overlaps the Cayley inverse
  float xr[8], sr[8];
  if (active) {
    if constexpr (!CHAINED) lds_row(xr, h + e * DD + 8 * r);  // generic load: h is read and written here
    const float4* sp = reinterpret_cast<const float4*>(S + e * DD + 8 * r);
    const float4 s0 = __ldg(sp), s1 = __ldg(sp + 1);
    sr[0] = s0.x; sr[1] = s0.y; sr[2] = s0.z; sr[3] = s0.w;
    sr[4] = s1.x; sr[5] = s1.y; sr[6] = s1.z; sr[7] = s1.w;
  } else {
#pragma unroll
    for (int c = 0; c < 8; ++c) xr[c] = sr[c] = 0.0f;
  }
  const float dtv = active ? __ldg(dt + b) : 0.0f;
  const float hdt = 0.5f * dtv;
  float row[8];  // row r of E = A - I (the deviation form of gj_inverse_dev)
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    if (c == r) {
      row[c] = 0.0f;
    } else {
      const int u = c < r ? c : r, v = c < r ? r : c;
      const int k = u * 8 - u * (u + 1) / 2 + (v - u - 1);
      const float w = active ? hdt * __ldg(gens + e * K + k) : 0.0f;
      row[c] = c < r ? w : -w;
    }
  }
  // Gauss-Jordan without pivoting (every pivot of I - Omega is >= 1), in the deviation
  // form of gj_inverse_dev: rows end as those of (I - Omega)^{-1} - I
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    float p[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) p[c] = __shfl_sync(FULL, row[c], k, 8);
    const float inv = 1.0f / (1.0f + p[k]);
#pragma unroll
    for (int c = 0; c < 8; ++c) p[c] = (c == k) ? -p[k] * inv : p[c] * inv;
    if (r == k) {
#pragma unroll
      for (int c = 0; c < 8; ++c) row[c] = p[c];
    } else {
      const float f = row[k];
#pragma unroll
      for (int c = 0; c < 8; ++c)
        if (c != k) row[c] = fmaf(-f, p[c], row[c]);
      row[k] = -f * inv;
    }
  }
  float alpha = 1.0f, sa = 1.0f;
  if constexpr (DAMPED) {
    if (active) {
      alpha = 1.0f / (1.0f + expf(__ldg(gamma + e) * dtv));
      sa = sqrtf(alpha);
    }
  }
#pragma unroll
  for (int c = 0; c < 8; ++c) row[c] = sa * fmaf(2.0f, row[c], (c == r) ? 1.0f : 0.0f);
  if constexpr (CHAINED) {
    asm volatile("griddepcontrol.wait;" ::: "memory");  // the previous step's state is complete
    if (active) lds_row(xr, h + e * DD + 8 * r);
  }
  sts_row(&sX[grp][8 * r], xr);
  sts_row(&sM[grp][8 * r], row);
  __syncwarp();
  // Y = M X: row r of Y = sum_k M[r][k] X[k][:]
  float y[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) y[c] = 0.0f;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    float xk[8];
    lds_row(xk, &sX[grp][8 * k]);
#pragma unroll
    for (int c = 0; c < 8; ++c) y[c] = fmaf(row[k], xk[c], y[c]);
  }
  if constexpr (TWO) {  // Z = Y M^T: Z[r][l] = sum_j Y[r][j] M[l][j]
    float z[8];
#pragma unroll
    for (int l = 0; l < 8; ++l) {
      float ml[8];
      lds_row(ml, &sM[grp][8 * l]);
      float acc = 0.0f;
#pragma unroll
      for (int j = 0; j < 8; ++j) acc = fmaf(y[j], ml[j], acc);
      z[l] = acc;
    }
#pragma unroll
    for (int c = 0; c < 8; ++c) y[c] = z[c];
  }
  if (!active) return;
  const float cs = DAMPED ? (1.0f - alpha) : 1.0f;
#pragma unroll
  for (int c = 0; c < 8; ++c) y[c] = fmaf(cs, sr[c], y[c]);
  sts_row(h + e * DD + 8 * r, y);
}

template <bool DAMPED, bool TWO>
int run_step8(const float* gens, const float* dt, const float* gamma, const float* S, float* h,
              int64_t B, int64_t N, bool chained, cudaStream_t st) {
  const int64_t states = B * N;
  const unsigned grid = (unsigned)((states + STEP_THREADS / 8 - 1) / (STEP_THREADS / 8));
  KernelTimer kt("rotor_step", st);
  if (!chained) {
    step8_kernel<DAMPED, TWO, false><<<grid, STEP_THREADS, 0, st>>>(gens, dt, gamma, S, h, B, N);
    return check_launch("rotor step (D=8)");
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(STEP_THREADS);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t err = cudaLaunchKernelEx(&cfg, step8_kernel<DAMPED, TWO, true>, gens, dt, gamma, S, h, B, N);
  if (err != cudaSuccess) return set_cuda_error(err, "rotor step (D=8, chained): cudaLaunchKernelEx");
  return check_launch("rotor step (D=8, chained)");
}

}  // namespace s8

int scan8_rotor_dispatch(const ScanArgs& a, bool damped, bool two, bool bwd, cudaStream_t st) {
  using namespace s8;
  if (damped) return two ? run8<true, true>(a, bwd, st) : run8<true, false>(a, bwd, st);
  return two ? run8<false, true>(a, bwd, st) : run8<false, false>(a, bwd, st);
}

int scan8_rotor_step(const float* gens, const float* dt, const float* gamma, const float* S, float* h,
                     int64_t B, int64_t N, bool two, bool chained, cudaStream_t st) {
  using namespace s8;
  if (gamma) return two ? run_step8<true, true>(gens, dt, gamma, S, h, B, N, chained, st)
                        : run_step8<true, false>(gens, dt, gamma, S, h, B, N, chained, st);
  return two ? run_step8<false, true>(gens, dt, gamma, S, h, B, N, chained, st)
             : run_step8<false, false>(gens, dt, gamma, S, h, B, N, chained, st);
}

}  // namespace csn
