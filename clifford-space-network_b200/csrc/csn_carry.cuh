// csn_carry.cuh -- per-sequence carry propagation between time chunks, shared by
// the D = 4/8 and D = 16 scan families, and the shard-aggregate composition.
#pragma once

#include <type_traits>

#include "csn_common.cuh"
#include "csn_scan_args.cuh"

namespace csn {

// ------------------------------------------------------------ carries, D = 4
// One thread per sequence walks the chunk aggregates (D = 8 and 16 use the grouped
// carry below).  Forward: h_0 = h0, h_{j+1} = P_j h_j P_j^T + c_j (one-sided P_j h_j + c_j).
template <int D, bool TWO>
__global__ void __launch_bounds__(128) fwd_carry_kernel(ScanArgs a) {
  static_assert(D == 4, "thread-per-sequence carry is the D = 4 path");
  const int64_t S = a.B * a.N;
  const int64_t s = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (s >= S) return;
  Mat<4> h, P;
  if (a.h0) load_mat(h, a.h0 + s * 16); else mat_zero(h);
  store_mat(a.carry + (s * a.nchunks) * 16, h);
  for (int64_t j = 0; j + 1 < a.nchunks; ++j) {
    load_mat(P, a.aggP + (s * a.nchunks + j) * 16);
    lmul(P, h);
    if constexpr (TWO) rmulT(h, P);
    add_scaled_mat(h, a.aggC + (s * a.nchunks + j) * 16, 1.0f);
    store_mat(a.carry + (s * a.nchunks + j + 1) * 16, h);
  }
}

// Backward: H_{nchunks-1} = hT (or 0);  H_{j-1} = P_j^T H_j P_j + c'_j  (one-sided: P_j^T H_j + c'_j)
template <int D, bool TWO>
__global__ void __launch_bounds__(128) bwd_carry_kernel(ScanArgs a) {
  static_assert(D == 4, "thread-per-sequence carry is the D = 4 path");
  const int64_t S = a.B * a.N;
  const int64_t s = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (s >= S) return;
  Mat<4> H, P;
  if (a.hT) load_mat(H, a.hT + s * 16); else mat_zero(H);
  store_mat(a.carry + (s * a.nchunks + a.nchunks - 1) * 16, H);
  for (int64_t j = a.nchunks - 1; j >= 1; --j) {
    load_mat(P, a.aggP + (s * a.nchunks + j) * 16);
    lmulT(P, H);
    if constexpr (TWO) rmul(H, P);
    add_scaled_mat(H, a.aggC + (s * a.nchunks + j) * 16, 1.0f);
    store_mat(a.carry + (s * a.nchunks + j - 1) * 16, H);
  }
}

// ddt[b, t] = sum_n ddt_part[b, t, n]
static __global__ void reduce_channels_kernel(const float* __restrict__ part, float* __restrict__ out,
                                       int64_t BT, int64_t N) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= BT) return;
  const float* p = part + i * N;
  float s = 0.0f;
  if ((N & 3) == 0 && (reinterpret_cast<uintptr_t>(p) & 15u) == 0) {
    // the same left-to-right sum from 16-byte loads
    for (int64_t n = 0; n < N; n += 4) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(p + n));
      s += v.x;
      s += v.y;
      s += v.z;
      s += v.w;
    }
  } else {
    for (int64_t n = 0; n < N; ++n) s += p[n];
  }
  out[i] = s;
}

// ------------------------------------------------------------ shard aggregates
// Forward: fold the chunk aggregates of one sequence into the shard aggregate
//   (P, c) <- (P_j P, P_j c P_j^T + c_j)   (one-sided: P_j c + c_j),  j = 0 .. nchunks-1
// Backward (REVERSE): H <- P_j^T H P_j + c'_j for j = nchunks-1 .. 0, output H.
// One warp per sequence, lane l owns D*D/32 entries (D = 4: lanes 0..15 own one each).
template <int D, bool TWO, bool REVERSE>
__global__ void __launch_bounds__(128) compose_kernel(ScanArgs a) {
  constexpr int DD = D * D;
  constexpr int PER = DD >= 32 ? DD / 32 : 1;
  __shared__ float sh_h[4][DD];
  __shared__ float sh_P[4][DD];
  __shared__ float sh_acc[4][DD];
  __shared__ float sh_y[4][DD];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t s = blockIdx.x * 4 + w;
  if (s >= a.B * a.N) return;
  float* h = sh_h[w];
  float* P = sh_P[w];
  float* acc = sh_acc[w];  // running product (forward only)
  float* y = sh_y[w];
#pragma unroll
  for (int q = 0; q < PER; ++q) {
    const int idx = lane + 32 * q;
    if (idx < DD) {
      h[idx] = 0.0f;
      acc[idx] = (idx / D == idx % D) ? 1.0f : 0.0f;
    }
  }
  __syncwarp();
  for (int64_t k = 0; k < a.nchunks; ++k) {
    const int64_t j = REVERSE ? (a.nchunks - 1 - k) : k;
    float cv[PER];
#pragma unroll
    for (int q = 0; q < PER; ++q) {
      const int idx = lane + 32 * q;
      if (idx < DD) {
        P[idx] = a.aggP[(s * a.nchunks + j) * DD + idx];
        cv[q] = a.aggC[(s * a.nchunks + j) * DD + idx];
      }
    }
    __syncwarp();
#pragma unroll
    for (int q = 0; q < PER; ++q) {  // y = P h (forward) | P^T h (reverse)
      const int idx = lane + 32 * q, i = idx / D, jj = idx % D;
      if (idx < DD) {
        float v = 0.0f;
#pragma unroll
        for (int kk = 0; kk < D; ++kk) v = fmaf(REVERSE ? P[kk * D + i] : P[i * D + kk], h[kk * D + jj], v);
        y[idx] = v;
      }
    }
    __syncwarp();
    float nv[PER], na[PER];
#pragma unroll
    for (int q = 0; q < PER; ++q) {
      const int idx = lane + 32 * q, i = idx / D, l = idx % D;
      if (idx < DD) {
        float v;
        if (TWO) {  // y P^T (forward) | y P (reverse)
          v = 0.0f;
#pragma unroll
          for (int kk = 0; kk < D; ++kk) v = fmaf(y[i * D + kk], REVERSE ? P[kk * D + l] : P[l * D + kk], v);
        } else {
          v = y[idx];
        }
        nv[q] = v + cv[q];
        if (!REVERSE) {  // running product P_j acc
          float p = 0.0f;
#pragma unroll
          for (int kk = 0; kk < D; ++kk) p = fmaf(P[i * D + kk], acc[kk * D + l], p);
          na[q] = p;
        }
      }
    }
    __syncwarp();
#pragma unroll
    for (int q = 0; q < PER; ++q) {
      const int idx = lane + 32 * q;
      if (idx < DD) {
        h[idx] = nv[q];
        if (!REVERSE) acc[idx] = na[q];
      }
    }
    __syncwarp();
  }
#pragma unroll
  for (int q = 0; q < PER; ++q) {
    const int idx = lane + 32 * q;
    if (idx < DD) {
      a.c_out[s * DD + idx] = h[idx];
      if (!REVERSE && a.P_out) a.P_out[s * DD + idx] = acc[idx];
    }
  }
}


// ------------------------------------------------------------ grouped carry (D = 16)
// The carry is a chain of links h <- L_k h L_k^T + c_k (one-sided: L_k h + c_k), one per
// chunk boundary: forward L_k = P_k, c_k = aggC_k, k = 0 .. nchunks-2, h_0 = h0; backward
// L_k = P_j^T, c_k = aggC_j with j = nchunks-1-k, h = hT at the last chunk.  One warp per
// sequence would walk it in nchunks-1 dependent links; here a block of W warps per sequence
// does it in about 2 (nchunks-1) / W + log2 W:
//   1. warp w composes its contiguous range of links into one link (L_w, c_w)
//   2. an inclusive scan of the W group links across the warps (log2 W levels), after which
//      (L_w, c_w) carries the state before group 0 to the state after group w
//   3. warp w takes its carry-in from group w - 1's prefix (no product when the initial
//      state is zero) and replays its range, writing every carry
// Composition of link 1 then link 2: (L2 L1, L2 c1 L2^T + c2)  (one-sided: L2 c1 + c2).
namespace carry_detail {

// Lane l owns the E = D*D/32 consecutive entries E*l .. E*l+E-1: columns c0 .. c0+E-1 of row
// i = l / (D/E), so every product below reads whole rows from shared memory with vector
// loads (rows of L, of m and, for the right-hand product, of L^T, staged beside L).
template <int D>
struct Lanes {
  static constexpr int E = D * D / 32, LPR = D / E;
};

template <int N>
__device__ __forceinline__ void ld(float (&v)[N], const float* p) {
  static_assert(N % 2 == 0, "pairs");
  if constexpr (N % 4 == 0) {
#pragma unroll
    for (int u = 0; u < N / 4; ++u) {
      const float4 f = *reinterpret_cast<const float4*>(p + 4 * u);
      v[4 * u] = f.x; v[4 * u + 1] = f.y; v[4 * u + 2] = f.z; v[4 * u + 3] = f.w;
    }
  } else {
#pragma unroll
    for (int u = 0; u < N / 2; ++u) {
      const float2 f = *reinterpret_cast<const float2*>(p + 2 * u);
      v[2 * u] = f.x; v[2 * u + 1] = f.y;
    }
  }
}
template <int N>
__device__ __forceinline__ void st(float* p, const float (&v)[N]) {
  if constexpr (N % 4 == 0) {
#pragma unroll
    for (int u = 0; u < N / 4; ++u)
      *reinterpret_cast<float4*>(p + 4 * u) = make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
  } else {
#pragma unroll
    for (int u = 0; u < N / 2; ++u) *reinterpret_cast<float2*>(p + 2 * u) = make_float2(v[2 * u], v[2 * u + 1]);
  }
}

// m <- L m L^T + c (one-sided: L m + c), warp-cooperative on shared memory; optionally
// Lacc <- L Lacc.  Lr holds L row-major, Lc holds L^T row-major; c holds this lane's entries.
template <int D, bool TWO, bool COMPOSE>
__device__ __forceinline__ void link_step(float* m, float* Lacc, const float* Lr, const float* Lc, float* y,
                                          const float (&c)[Lanes<D>::E], int lane) {
  constexpr int E = Lanes<D>::E, LPR = Lanes<D>::LPR;
  const int i = lane / LPR, c0 = E * (lane % LPR), o = E * lane;
  float lrow[D], acc[E], accL[E];
  ld<D>(lrow, Lr + i * D);
#pragma unroll
  for (int q = 0; q < E; ++q) acc[q] = accL[q] = 0.0f;
#pragma unroll
  for (int k = 0; k < D; ++k) {
    float mk[E];
    ld<E>(mk, m + k * D + c0);
#pragma unroll
    for (int q = 0; q < E; ++q) acc[q] = fmaf(lrow[k], mk[q], acc[q]);
    if (COMPOSE) {
      float lk[E];
      ld<E>(lk, Lacc + k * D + c0);
#pragma unroll
      for (int q = 0; q < E; ++q) accL[q] = fmaf(lrow[k], lk[q], accL[q]);
    }
  }
  float nv[E];
  if constexpr (TWO) {
    st<E>(y + o, acc);
    __syncwarp();
    float yrow[D];
    ld<D>(yrow, y + i * D);
#pragma unroll
    for (int q = 0; q < E; ++q) nv[q] = c[q];
#pragma unroll
    for (int k = 0; k < D; ++k) {
      float lk[E];
      ld<E>(lk, Lc + k * D + c0);  // (L^T)[k][c0 ..] = L[c0 ..][k]
#pragma unroll
      for (int q = 0; q < E; ++q) nv[q] = fmaf(yrow[k], lk[q], nv[q]);
    }
  } else {
#pragma unroll
    for (int q = 0; q < E; ++q) nv[q] = acc[q] + c[q];
  }
  __syncwarp();
  st<E>(m + o, nv);
  if (COMPOSE) st<E>(Lacc + o, accL);
  __syncwarp();
}

// Stage a link operator: Lr <- L (this lane's entries v), Lc <- L^T.
template <int D>
__device__ __forceinline__ void stage_link(float* Lr, float* Lc, const float (&v)[Lanes<D>::E], int lane) {
  constexpr int E = Lanes<D>::E, LPR = Lanes<D>::LPR;
  const int i = lane / LPR, c0 = E * (lane % LPR);
  st<E>(Lr + E * lane, v);
#pragma unroll
  for (int q = 0; q < E; ++q) Lc[(c0 + q) * D + i] = v[q];
}

}  // namespace carry_detail

// Most warps per sequence: 32 for D <= 8, 16 for D = 16 (its link state is 4x larger).
template <int D>
constexpr int carry_max_warps() { return D <= 8 ? 32 : 16; }

template <int D, bool TWO, bool REVERSE>
__global__ void __launch_bounds__(32 * carry_max_warps<D>()) carry_grouped_kernel(ScanArgs a) {
  using namespace carry_detail;
  constexpr int DD = D * D, E = Lanes<D>::E;
  extern __shared__ __align__(16) float cg_smem[];
  const int nw = blockDim.x >> 5, w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int o = E * lane;  // this lane's entries
  const int64_t s = blockIdx.x;
  const int64_t nch = a.nchunks, nl = nch - 1;
  const int64_t base = s * nch;
  float* m = cg_smem + (size_t)w * 5 * DD;  // warp's running matrix
  float* Lr = m + DD;                         // staged link operator L (rows)
  float* Lc = m + 2 * DD;                     // and its transpose
  float* Lx = m + 3 * DD;                     // scan scratch (an earlier prefix's operator)
  float* y = m + 4 * DD;                      // product scratch
  float* gL = cg_smem + (size_t)nw * 5 * DD;  // [nw][DD] group operators
  float* gC = gL + (size_t)nw * DD;           // [nw][DD] group offsets
  const int64_t per = (nl + nw - 1) / nw;
  const int64_t k0 = min(nl, (int64_t)w * per), k1 = min(nl, k0 + per);
  auto chunk_of = [&](int64_t k) { return REVERSE ? nch - 1 - k : k; };
  auto out_of = [&](int64_t k) { return REVERSE ? nch - 2 - k : k + 1; };

  // Walk links [k0, k1) on `m` (composing into gL[w] when COMPOSE).  The aggregates of the
  // next PF links are in flight while a link is applied (a ring of register slots, unrolled
  // so that slot indices are compile-time); a link's own work is far shorter than a load
  // from memory.  Backward links use P^T: the staged rows and columns swap.
  auto walk = [&](auto compose_tag) {
    constexpr bool COMPOSE = decltype(compose_tag)::value;
    constexpr int PF = D <= 8 ? 4 : 2;
    float pn[PF][E], cn[PF][E];
#pragma unroll
    for (int u = 0; u < PF; ++u)
      if (k0 + u < k1) {
        ld<E>(pn[u], a.aggP + (base + chunk_of(k0 + u)) * DD + o);
        ld<E>(cn[u], a.aggC + (base + chunk_of(k0 + u)) * DD + o);
      }
    for (int64_t kk = k0; kk < k1; kk += PF) {
#pragma unroll
      for (int u = 0; u < PF; ++u) {
        const int64_t k = kk + u;
        if (k >= k1) break;
        float cv[E];
        stage_link<D>(REVERSE ? Lc : Lr, REVERSE ? Lr : Lc, pn[u], lane);
#pragma unroll
        for (int q = 0; q < E; ++q) cv[q] = cn[u][q];
        if (k + PF < k1) {
          ld<E>(pn[u], a.aggP + (base + chunk_of(k + PF)) * DD + o);
          ld<E>(cn[u], a.aggC + (base + chunk_of(k + PF)) * DD + o);
        }
        __syncwarp();
        link_step<D, TWO, COMPOSE>(m, gL + (size_t)w * DD, Lr, Lc, y, cv, lane);
        if (!COMPOSE) {
          float mv[E];
          ld<E>(mv, m + o);
          st<E>(a.carry + (base + out_of(k)) * DD + o, mv);
        }
      }
    }
  };

  // 1. group links: m = c_w (from zero), gL[w] = L_w (from the identity)
  {
    float z[E], id[E];
#pragma unroll
    for (int q = 0; q < E; ++q) {
      z[q] = 0.0f;
      id[q] = ((o + q) / D == (o + q) % D) ? 1.0f : 0.0f;
    }
    st<E>(m + o, z);
    st<E>(gL + (size_t)w * DD + o, id);
  }
  __syncwarp();
  walk(std::integral_constant<bool, true>{});
  {
    float mv[E];
    ld<E>(mv, m + o);
    st<E>(gC + (size_t)w * DD + o, mv);
  }
  __syncthreads();
  // 2. inclusive scan of the group links (Hillis-Steele): at distance d, warp w >= d puts the
  //    prefix of group w - d before its own.  Read, compose and write are separated by block
  //    barriers, so no warp overwrites a prefix another warp still reads.
  for (int d = 1; d < nw; d <<= 1) {
    const bool act = w >= d;
    float cv[E];
    if (act) {
      float v[E];
      ld<E>(v, gC + (size_t)(w - d) * DD + o);
      st<E>(m + o, v);
      ld<E>(v, gL + (size_t)(w - d) * DD + o);
      st<E>(Lx + o, v);
      ld<E>(v, gL + (size_t)w * DD + o);
      stage_link<D>(Lr, Lc, v, lane);
      ld<E>(cv, gC + (size_t)w * DD + o);
    }
    __syncthreads();
    if (act) link_step<D, TWO, true>(m, Lx, Lr, Lc, y, cv, lane);
    __syncthreads();
    if (act) {
      float v[E];
      ld<E>(v, m + o);
      st<E>(gC + (size_t)w * DD + o, v);
      ld<E>(v, Lx + o);
      st<E>(gL + (size_t)w * DD + o, v);
    }
    __syncthreads();
  }
  // 3. carry-in of group w: the initial state carried through groups 0 .. w-1; then replay
  const float* init = REVERSE ? a.hT : a.h0;
  {
    float v[E];
    if (init) ld<E>(v, init + s * DD + o);
    else {
#pragma unroll
      for (int q = 0; q < E; ++q) v[q] = 0.0f;
    }
    if (w == 0) st<E>(a.carry + (base + (REVERSE ? nch - 1 : 0)) * DD + o, v);
    if (w > 0 && !init) ld<E>(v, gC + (size_t)(w - 1) * DD + o);
    st<E>(m + o, v);
  }
  if (w > 0 && init) {
    float v[E], cv[E];
    ld<E>(v, gL + (size_t)(w - 1) * DD + o);
    stage_link<D>(Lr, Lc, v, lane);
    ld<E>(cv, gC + (size_t)(w - 1) * DD + o);
    __syncwarp();
    link_step<D, TWO, false>(m, nullptr, Lr, Lc, y, cv, lane);
  }
  __syncwarp();
  walk(std::integral_constant<bool, false>{});
}

// ------------------------------------------------ grouped carry on fp64 MMA (D = 8)
// The same three phases as carry_grouped_kernel, with every 8 x 8 product on the FP64 tensor
// cores (mma.sync m8n8k4 f64) instead of shared-memory round trips: a warp holds a matrix as
// the m8n8k4 accumulator fragment, lane 4 r + c owning X[r][2c] and X[r][2c+1].  Read with
// the k-steps taking the even columns, then the odd ones, the same fragment is also the A
// operand of X and the B operand of X^T, so nt(A, Y, C) = A Y^T + C needs no data movement.
//   link (two-sided):  w = nt(L, m, 0) = L m^T,  m' = nt(L, w, c) = L m L^T + c
//   link (one-sided):  the state is held transposed, m'^T = nt(m^T, L, c^T) = (L m + c)^T
//   group operator:    G^T <- nt(G^T, L, 0) = (L G)^T
// Links and states are carried in fp64 (the chunk aggregates are read as float); each carry
// is written as the float nearest to it.
namespace carry8 {

struct Frag {
  double x0, x1;
};

__device__ __forceinline__ void dmma(double& d0, double& d1, double a, double b) {
  asm("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0,%1}, {%2}, {%3}, {%0,%1};\n"
      : "+d"(d0), "+d"(d1)
      : "d"(a), "d"(b));
}

__device__ __forceinline__ Frag nt(const Frag& A, const Frag& Y, Frag C) {
  dmma(C.x0, C.x1, A.x0, Y.x0);
  dmma(C.x0, C.x1, A.x1, Y.x1);
  return C;
}

__device__ __forceinline__ Frag zero() { return Frag{0.0, 0.0}; }
__device__ __forceinline__ Frag identity(int r, int c) {
  return Frag{(r == 2 * c) ? 1.0 : 0.0, (r == 2 * c + 1) ? 1.0 : 0.0};
}

// fragment of X (T = false) or of X^T (T = true) from a row-major 8 x 8 array
template <bool T, typename F>
__device__ __forceinline__ Frag load(const F* p, int r, int c) {
  if constexpr (T) return Frag{(double)p[(2 * c) * 8 + r], (double)p[(2 * c + 1) * 8 + r]};
  else return Frag{(double)p[r * 8 + 2 * c], (double)p[r * 8 + 2 * c + 1]};
}
template <bool T, typename F>
__device__ __forceinline__ void store(F* p, const Frag& X, int r, int c) {
  if constexpr (T) {
    p[(2 * c) * 8 + r] = (F)X.x0;
    p[(2 * c + 1) * 8 + r] = (F)X.x1;
  } else {
    p[r * 8 + 2 * c] = (F)X.x0;
    p[r * 8 + 2 * c + 1] = (F)X.x1;
  }
}

// one link on the state: two-sided m <- L m L^T + c, one-sided (state transposed) m^T <- m^T L^T + c^T
template <bool TWO>
__device__ __forceinline__ Frag link(const Frag& L, const Frag& m, const Frag& c) {
  if constexpr (TWO) return nt(L, nt(L, m, zero()), c);
  else return nt(m, L, c);
}

}  // namespace carry8

// Most warps per sequence and links per warp of the fp64-MMA carry.
constexpr int CARRY8_MAX_WARPS = 16;
constexpr int CARRY8_LINKS_PER_WARP = 16;

template <bool TWO, bool REVERSE>
__global__ void __launch_bounds__(32 * CARRY8_MAX_WARPS) carry8_mma_kernel(ScanArgs a) {
  using namespace carry8;
  constexpr int DD = 64;
  // the operator and the offset of every warp's group, in fp64: [nw][DD] each
  extern __shared__ __align__(16) double c8_smem[];
  const int nw = blockDim.x >> 5, w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = lane >> 2, c = lane & 3;
  const int64_t s = blockIdx.x;
  const int64_t nch = a.nchunks, nl = nch - 1;
  const int64_t base = s * nch;
  double* gG = c8_smem;                      // group operators G_w, row-major
  double* gC = c8_smem + (size_t)nw * DD;    // group offsets (the state's own orientation)
  const int64_t per = (nl + nw - 1) / nw;
  const int64_t k0 = min(nl, (int64_t)w * per), k1 = min(nl, k0 + per);
  // link k: forward L = P_k, c = aggC_k, writes carry k + 1;  backward (chunk j = nch-1-k)
  // L = P_j^T, c = aggC_j, writes carry j - 1.  One-sided states are held transposed.
  auto chunk_of = [&](int64_t k) { return REVERSE ? nch - 1 - k : k; };
  auto out_of = [&](int64_t k) { return REVERSE ? nch - 2 - k : k + 1; };
  // the lane's two entries of a link's L and c fragments, as stored (float)
  auto load_link = [&](int64_t k, float (&v)[4]) {
    const float* P = a.aggP + (base + chunk_of(k)) * DD;
    const float* C = a.aggC + (base + chunk_of(k)) * DD;
    const int lo = REVERSE ? (2 * c) * 8 + r : r * 8 + 2 * c, lstep = REVERSE ? 8 : 1;
    const int co = TWO ? r * 8 + 2 * c : (2 * c) * 8 + r, cstep = TWO ? 1 : 8;
    v[0] = __ldg(P + lo);
    v[1] = __ldg(P + lo + lstep);
    v[2] = __ldg(C + co);
    v[3] = __ldg(C + co + cstep);
  };

  // Walk links [k0, k1), composing G^T when COMPOSE and writing every carry otherwise; the
  // next PF links' operands are in flight meanwhile (a ring of register slots, unrolled so
  // that slot indices are compile-time).
  constexpr int PF = 4;
  auto walk = [&](auto compose_tag, Frag& m, Frag& T) {
    constexpr bool COMPOSE = decltype(compose_tag)::value;
    float ring[PF][4];
#pragma unroll
    for (int u = 0; u < PF; ++u)
      if (k0 + u < k1) load_link(k0 + u, ring[u]);
    for (int64_t kk = k0; kk < k1; kk += PF) {
#pragma unroll
      for (int u = 0; u < PF; ++u) {
        const int64_t k = kk + u;
        if (k >= k1) break;
        const Frag L{(double)ring[u][0], (double)ring[u][1]};
        const Frag cf{(double)ring[u][2], (double)ring[u][3]};
        if (k + PF < k1) load_link(k + PF, ring[u]);
        m = link<TWO>(L, m, cf);
        if constexpr (COMPOSE) T = nt(T, L, zero());
        else store<!TWO>(a.carry + (base + out_of(k)) * DD, m, r, c);
      }
    }
  };

  // 1. group links: (G_w, c_w) composed from the identity and a zero state
  {
    Frag m = zero(), T = identity(r, c);
    walk(std::integral_constant<bool, true>{}, m, T);
    store<true>(gG + (size_t)w * DD, T, r, c);  // G_w from G_w^T
    store<!TWO>(gC + (size_t)w * DD, m, r, c);
  }
  __syncthreads();
  // 2. inclusive scan of the group links (Hillis-Steele): at distance d, warp w >= d puts the
  //    prefix of group w - d before its own: c <- G_w c_p G_w^T + c_w (one-sided G_w c_p +
  //    c_w), G <- G_w G_p.  Reads and writes are separated by block barriers.
  for (int d = 1; d < nw; d <<= 1) {
    const bool act = w >= d;
    Frag mn, Tn;
    if (act) {
      const Frag L = load<false>(gG + (size_t)w * DD, r, c);
      const Frag Tp = load<true>(gG + (size_t)(w - d) * DD, r, c);
      const Frag mp = load<!TWO>(gC + (size_t)(w - d) * DD, r, c);
      const Frag cw = load<!TWO>(gC + (size_t)w * DD, r, c);
      mn = link<TWO>(L, mp, cw);
      Tn = nt(Tp, L, zero());
    }
    __syncthreads();
    if (act) {
      store<true>(gG + (size_t)w * DD, Tn, r, c);
      store<!TWO>(gC + (size_t)w * DD, mn, r, c);
    }
    __syncthreads();
  }
  // 3. carry-in of group w: the initial state carried through groups 0 .. w-1; then replay
  const float* init = REVERSE ? a.hT : a.h0;
  Frag m = init ? load<!TWO>(init + s * DD, r, c) : zero();
  if (w == 0) store<!TWO>(a.carry + (base + (REVERSE ? nch - 1 : 0)) * DD, m, r, c);
  if (w > 0) {
    const Frag cp = load<!TWO>(gC + (size_t)(w - 1) * DD, r, c);
    if (init) m = link<TWO>(load<false>(gG + (size_t)(w - 1) * DD, r, c), m, cp);
    else m = cp;
  }
  Frag unused = zero();
  walk(std::integral_constant<bool, false>{}, m, unused);
}

// Shard aggregate of one sequence from its chunk aggregates (the compose_kernel contract):
// forward (P, c) <- (P_j P, P_j c P_j^T + c_j) over j = 0 .. nchunks-1 from (I, 0), written to
// P_out (if set) and c_out; backward H <- P_j^T H P_j + c'_j over j = nchunks-1 .. 0 from 0,
// written to c_out.  Phases 1 and 2 of carry8_mma_kernel over all nchunks links; the last
// warp's inclusive prefix is the whole composition.
template <bool TWO, bool REVERSE>
__global__ void __launch_bounds__(32 * CARRY8_MAX_WARPS) compose8_mma_kernel(ScanArgs a) {
  using namespace carry8;
  constexpr int DD = 64;
  extern __shared__ __align__(16) double c8_smem[];
  const int nw = blockDim.x >> 5, w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = lane >> 2, c = lane & 3;
  const int64_t s = blockIdx.x;
  const int64_t nch = a.nchunks, nl = nch;
  const int64_t base = s * nch;
  double* gG = c8_smem;
  double* gC = c8_smem + (size_t)nw * DD;
  const int64_t per = (nl + nw - 1) / nw;
  const int64_t k0 = min(nl, (int64_t)w * per), k1 = min(nl, k0 + per);
  Frag m = zero(), T = identity(r, c);
  for (int64_t k = k0; k < k1; ++k) {
    const int64_t j = REVERSE ? nch - 1 - k : k;
    const Frag L = load<REVERSE>(a.aggP + (base + j) * DD, r, c);
    const Frag cf = load<!TWO>(a.aggC + (base + j) * DD, r, c);
    m = link<TWO>(L, m, cf);
    T = nt(T, L, zero());
  }
  store<true>(gG + (size_t)w * DD, T, r, c);
  store<!TWO>(gC + (size_t)w * DD, m, r, c);
  __syncthreads();
  for (int d = 1; d < nw; d <<= 1) {
    const bool act = w >= d;
    Frag mn, Tn;
    if (act) {
      const Frag L = load<false>(gG + (size_t)w * DD, r, c);
      const Frag Tp = load<true>(gG + (size_t)(w - d) * DD, r, c);
      const Frag mp = load<!TWO>(gC + (size_t)(w - d) * DD, r, c);
      const Frag cw = load<!TWO>(gC + (size_t)w * DD, r, c);
      mn = link<TWO>(L, mp, cw);
      Tn = nt(Tp, L, zero());
    }
    __syncthreads();
    if (act) {
      store<true>(gG + (size_t)w * DD, Tn, r, c);
      store<!TWO>(gC + (size_t)w * DD, mn, r, c);
    }
    __syncthreads();
  }
  if (w == nw - 1) {
    store<!TWO>(a.c_out + s * DD, load<!TWO>(gC + (size_t)w * DD, r, c), r, c);
    if (!REVERSE && a.P_out) store<false>(a.P_out + s * DD, load<false>(gG + (size_t)w * DD, r, c), r, c);
  }
}

template <bool TWO, bool REVERSE>
inline void launch_compose8_mma(const ScanArgs& a, cudaStream_t st) {
  int64_t w = (a.nchunks + CARRY8_LINKS_PER_WARP - 1) / CARRY8_LINKS_PER_WARP;
  w = w < 1 ? 1 : w > CARRY8_MAX_WARPS ? CARRY8_MAX_WARPS : w;
  const size_t smem = (size_t)2 * w * 64 * sizeof(double);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(compose8_mma_kernel<TWO, REVERSE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
  compose8_mma_kernel<TWO, REVERSE><<<(unsigned)(a.B * a.N), 32 * (unsigned)w, smem, st>>>(a);
}

template <bool TWO, bool REVERSE>
inline void launch_carry8_mma(const ScanArgs& a, cudaStream_t st) {
  const int64_t nl = a.nchunks - 1;
  int64_t w = (nl + CARRY8_LINKS_PER_WARP - 1) / CARRY8_LINKS_PER_WARP;
  w = w < 1 ? 1 : w > CARRY8_MAX_WARPS ? CARRY8_MAX_WARPS : w;
  const size_t smem = (size_t)2 * w * 64 * sizeof(double);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(carry8_mma_kernel<TWO, REVERSE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
  carry8_mma_kernel<TWO, REVERSE><<<(unsigned)(a.B * a.N), 32 * (unsigned)w, smem, st>>>(a);
}

// Warps per sequence for the grouped carry: about 16 links per warp.
template <int D>
inline int carry_warps(int64_t nchunks) {
  const int64_t nl = nchunks - 1;
  int64_t w = (nl + 15) / 16;
  return (int)(w < 1 ? 1 : w > carry_max_warps<D>() ? carry_max_warps<D>() : w);
}

template <int D>
inline size_t carry_smem_bytes(int warps) { return (size_t)7 * warps * D * D * sizeof(float); }

// Launch the carry pass of a chunked scan (nchunks > 1): fp64 MMA for D = 8, grouped on
// shared memory for D = 16.
template <int D, bool TWO, bool REVERSE>
inline void launch_grouped_carry(const ScanArgs& a, cudaStream_t st) {
  if constexpr (D == 8) {
    launch_carry8_mma<TWO, REVERSE>(a, st);
    return;
  }
  const int w = carry_warps<D>(a.nchunks);
  const size_t smem = carry_smem_bytes<D>(w);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(carry_grouped_kernel<D, TWO, REVERSE>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  carry_grouped_kernel<D, TWO, REVERSE><<<(unsigned)(a.B * a.N), 32 * w, smem, st>>>(a);
}

}  // namespace csn
