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
// sequence walks it serially in nchunks-1 dependent links; here a block of W warps per
// sequence does it in about 2 (nchunks-1) / W + W:
//   1. warp w composes its contiguous range of links into one link (L_w, c_w)
//   2. warp 0 walks the W group links from the initial state -> carry-in of every group
//   3. warp w replays its range from its carry-in, writing every carry
// Composition of link 1 then link 2: (L2 L1, L2 c1 L2^T + c2)  (one-sided: L2 c1 + c2).
namespace carry_detail {

// y = op(L) m, with op(L) = L or, for TR, the transpose of the matrix stored at Lm.
template <int D, bool TR>
__device__ __forceinline__ float left_entry(const float* Lm, const float* m, int i, int jj) {
  float acc = 0.0f;
#pragma unroll
  for (int k = 0; k < D; ++k) acc = fmaf(TR ? Lm[k * D + i] : Lm[i * D + k], m[k * D + jj], acc);
  return acc;
}

// (y op(L)^T)[i][l]
template <int D, bool TR>
__device__ __forceinline__ float right_entry(const float* y, const float* Lm, int i, int l) {
  float acc = 0.0f;
#pragma unroll
  for (int k = 0; k < D; ++k) acc = fmaf(y[i * D + k], TR ? Lm[k * D + l] : Lm[l * D + k], acc);
  return acc;
}

// m <- op(L) m op(L)^T + c  (one-sided: op(L) m + c), warp-cooperative on shared memory;
// optionally Lacc <- op(L) Lacc.  c holds this lane's entries lane + 32 q.
template <int D, bool TWO, bool TR, bool COMPOSE>
__device__ __forceinline__ void link_step(float* m, float* Lacc, const float* Lm, float* y,
                                          const float (&c)[D * D / 32], int lane) {
  constexpr int DD = D * D, PER = DD / 32;
  float ln[PER];
#pragma unroll
  for (int q = 0; q < PER; ++q) {
    const int idx = lane + 32 * q, i = idx / D, jj = idx % D;
    y[idx] = left_entry<D, TR>(Lm, m, i, jj);
    if (COMPOSE) ln[q] = left_entry<D, TR>(Lm, Lacc, i, jj);
  }
  __syncwarp();
  float nv[PER];
#pragma unroll
  for (int q = 0; q < PER; ++q) {
    const int idx = lane + 32 * q, i = idx / D, l = idx % D;
    nv[q] = (TWO ? right_entry<D, TR>(y, Lm, i, l) : y[idx]) + c[q];
  }
  __syncwarp();
#pragma unroll
  for (int q = 0; q < PER; ++q) {
    m[lane + 32 * q] = nv[q];
    if (COMPOSE) Lacc[lane + 32 * q] = ln[q];
  }
  __syncwarp();
}

}  // namespace carry_detail

template <int D, bool TWO, bool REVERSE>
__global__ void __launch_bounds__(512) carry_grouped_kernel(ScanArgs a) {
  using namespace carry_detail;
  constexpr int DD = D * D, PER = DD / 32;
  extern __shared__ __align__(16) float cg_smem[];
  const int nw = blockDim.x >> 5, w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t s = blockIdx.x;
  const int64_t nch = a.nchunks, nl = nch - 1;
  const int64_t base = s * nch;
  float* m = cg_smem + (size_t)w * 3 * DD;  // warp's running matrix
  float* Lm = m + DD;                         // staged aggregate of the current link
  float* y = m + 2 * DD;                      // product scratch
  float* gL = cg_smem + (size_t)nw * 3 * DD;  // [nw][DD] group operators
  float* gC = gL + (size_t)nw * DD;           // [nw][DD] group offsets
  float* gH = gC + (size_t)nw * DD;           // [nw][DD] group carry-ins
  const int64_t per = (nl + nw - 1) / nw;
  const int64_t k0 = min(nl, (int64_t)w * per), k1 = min(nl, k0 + per);
  auto chunk_of = [&](int64_t k) { return REVERSE ? nch - 1 - k : k; };
  auto out_of = [&](int64_t k) { return REVERSE ? nch - 2 - k : k + 1; };

  // Walk links [k0, k1) on `m` (composing into gL[w] when COMPOSE), the next link's
  // aggregate loaded while the current one is applied.
  auto walk = [&](auto compose_tag) {
    constexpr bool COMPOSE = decltype(compose_tag)::value;
    float pn[PER], cn[PER];
    if (k0 < k1) {
#pragma unroll
      for (int q = 0; q < PER; ++q) {
        pn[q] = a.aggP[(base + chunk_of(k0)) * DD + lane + 32 * q];
        cn[q] = a.aggC[(base + chunk_of(k0)) * DD + lane + 32 * q];
      }
    }
    for (int64_t k = k0; k < k1; ++k) {
      float cv[PER];
#pragma unroll
      for (int q = 0; q < PER; ++q) {
        Lm[lane + 32 * q] = pn[q];
        cv[q] = cn[q];
      }
      if (k + 1 < k1) {
#pragma unroll
        for (int q = 0; q < PER; ++q) {
          pn[q] = a.aggP[(base + chunk_of(k + 1)) * DD + lane + 32 * q];
          cn[q] = a.aggC[(base + chunk_of(k + 1)) * DD + lane + 32 * q];
        }
      }
      __syncwarp();
      link_step<D, TWO, REVERSE, COMPOSE>(m, gL + (size_t)w * DD, Lm, y, cv, lane);
      if (!COMPOSE) {
#pragma unroll
        for (int q = 0; q < PER; ++q) a.carry[(base + out_of(k)) * DD + lane + 32 * q] = m[lane + 32 * q];
      }
    }
  };

  // 1. group links: m = c_w (from zero), gL[w] = L_w (from the identity)
#pragma unroll
  for (int q = 0; q < PER; ++q) {
    const int idx = lane + 32 * q;
    m[idx] = 0.0f;
    gL[(size_t)w * DD + idx] = (idx / D == idx % D) ? 1.0f : 0.0f;
  }
  __syncwarp();
  walk(std::integral_constant<bool, true>{});
#pragma unroll
  for (int q = 0; q < PER; ++q) gC[(size_t)w * DD + lane + 32 * q] = m[lane + 32 * q];
  __syncthreads();
  // 2. warp 0: carry-in of every group
  if (w == 0) {
    const float* init = REVERSE ? a.hT : a.h0;
#pragma unroll
    for (int q = 0; q < PER; ++q) {
      const int idx = lane + 32 * q;
      const float v = init ? init[s * DD + idx] : 0.0f;
      m[idx] = v;
      a.carry[(base + (REVERSE ? nch - 1 : 0)) * DD + idx] = v;
    }
    __syncwarp();
    for (int g = 0; g < nw; ++g) {
      float cv[PER];
#pragma unroll
      for (int q = 0; q < PER; ++q) {
        const int idx = lane + 32 * q;
        gH[(size_t)g * DD + idx] = m[idx];
        Lm[idx] = gL[(size_t)g * DD + idx];
        cv[q] = gC[(size_t)g * DD + idx];
      }
      __syncwarp();
      // group operators are already oriented (no transpose); an empty group is the identity
      link_step<D, TWO, false, false>(m, nullptr, Lm, y, cv, lane);
    }
  }
  __syncthreads();
  // 3. replay each range from its carry-in
#pragma unroll
  for (int q = 0; q < PER; ++q) m[lane + 32 * q] = gH[(size_t)w * DD + lane + 32 * q];
  __syncwarp();
  walk(std::integral_constant<bool, false>{});
}

// Warps per sequence for the grouped carry: about 8 links per warp, at most 16 warps.
inline int carry_warps(int64_t nchunks) {
  const int64_t nl = nchunks - 1;
  int64_t w = (nl + 7) / 8;
  return (int)(w < 1 ? 1 : w > 16 ? 16 : w);
}

template <int D>
inline size_t carry_smem_bytes(int warps) { return (size_t)6 * warps * D * D * sizeof(float); }

// Launch the carry pass of a chunked scan (nchunks > 1): grouped for D = 8, 16.
template <int D, bool TWO, bool REVERSE>
inline void launch_grouped_carry(const ScanArgs& a, cudaStream_t st) {
  const int w = carry_warps(a.nchunks);
  const size_t smem = carry_smem_bytes<D>(w);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(carry_grouped_kernel<D, TWO, REVERSE>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  carry_grouped_kernel<D, TWO, REVERSE><<<(unsigned)(a.B * a.N), 32 * w, smem, st>>>(a);
}

}  // namespace csn
