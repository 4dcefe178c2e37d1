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
  float s = 0.0f;
  for (int64_t n = 0; n < N; ++n) s += part[i * N + n];
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


// ------------------------------------------------------------ grouped carry (D = 8, 16)
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

// Warps per sequence for the grouped carry: about 16 links per warp.
template <int D>
inline int carry_warps(int64_t nchunks) {
  const int64_t nl = nchunks - 1;
  int64_t w = (nl + 15) / 16;
  return (int)(w < 1 ? 1 : w > carry_max_warps<D>() ? carry_max_warps<D>() : w);
}

template <int D>
inline size_t carry_smem_bytes(int warps) { return (size_t)7 * warps * D * D * sizeof(float); }

// Launch the carry pass of a chunked scan (nchunks > 1): grouped for D = 8, 16.
template <int D, bool TWO, bool REVERSE>
inline void launch_grouped_carry(const ScanArgs& a, cudaStream_t st) {
  const int w = carry_warps<D>(a.nchunks);
  const size_t smem = carry_smem_bytes<D>(w);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(carry_grouped_kernel<D, TWO, REVERSE>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  carry_grouped_kernel<D, TWO, REVERSE><<<(unsigned)(a.B * a.N), 32 * w, smem, st>>>(a);
}

}  // namespace csn
