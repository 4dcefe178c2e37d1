// csn_carry.cuh -- per-sequence carry propagation between time chunks, shared by
// the D = 4/8 and D = 16 scan families.
#pragma once

#include "csn_common.cuh"
#include "csn_scan_args.cuh"

namespace csn {

// ------------------------------------------------------------ forward: carry
// One warp per sequence; lane l owns D*D/32 entries (D = 8: 2, D = 16: 8) of the
// running carry.  D = 4 uses one thread per sequence.
template <int D, bool TWO>
__global__ void __launch_bounds__(128) fwd_carry_kernel(ScanArgs a) {
  const int64_t S = a.B * a.N;
  if constexpr (D == 4) {
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
  } else {
    constexpr int DD = D * D;
    constexpr int PER = DD / 32;
    __shared__ float sh_h[4][DD];
    __shared__ float sh_P[4][DD];
    __shared__ float sh_y[4][DD];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t s = blockIdx.x * 4 + w;
    if (s >= S) return;  // whole warp exits together
    float* h = sh_h[w];
    float* P = sh_P[w];
    float* y = sh_y[w];
#pragma unroll
    for (int q = 0; q < PER; ++q) {
      const int idx = lane + 32 * q;
      h[idx] = a.h0 ? a.h0[s * DD + idx] : 0.0f;
      a.carry[(s * a.nchunks) * DD + idx] = h[idx];
    }
    __syncwarp();
    // the aggregate of chunk j + 1 is loaded while chunk j's link is computed, so the
    // serial chain never waits on global memory
    float pn[PER], cn[PER];
#pragma unroll
    for (int q = 0; q < PER; ++q) {
      pn[q] = (a.nchunks > 1) ? a.aggP[(s * a.nchunks) * DD + lane + 32 * q] : 0.0f;
      cn[q] = (a.nchunks > 1) ? a.aggC[(s * a.nchunks) * DD + lane + 32 * q] : 0.0f;
    }
    for (int64_t j = 0; j + 1 < a.nchunks; ++j) {
      float cv[PER];
#pragma unroll
      for (int q = 0; q < PER; ++q) {
        P[lane + 32 * q] = pn[q];
        cv[q] = cn[q];
      }
      if (j + 2 < a.nchunks) {
#pragma unroll
        for (int q = 0; q < PER; ++q) {
          pn[q] = a.aggP[(s * a.nchunks + j + 1) * DD + lane + 32 * q];
          cn[q] = a.aggC[(s * a.nchunks + j + 1) * DD + lane + 32 * q];
        }
      }
      __syncwarp();
      // y = P h
#pragma unroll
      for (int q = 0; q < PER; ++q) {
        const int idx = lane + 32 * q, i = idx / D, jj = idx % D;
        float acc = 0.0f;
#pragma unroll
        for (int k = 0; k < D; ++k) acc = fmaf(P[i * D + k], h[k * D + jj], acc);
        y[idx] = acc;
      }
      __syncwarp();
      float nv[PER];
#pragma unroll
      for (int q = 0; q < PER; ++q) {
        const int idx = lane + 32 * q, i = idx / D, l = idx % D;
        float acc;
        if constexpr (TWO) {
          acc = 0.0f;
#pragma unroll
          for (int k = 0; k < D; ++k) acc = fmaf(y[i * D + k], P[l * D + k], acc);
        } else {
          acc = y[idx];
        }
        nv[q] = acc + cv[q];
      }
      __syncwarp();
#pragma unroll
      for (int q = 0; q < PER; ++q) {
        const int idx = lane + 32 * q;
        h[idx] = nv[q];
        a.carry[(s * a.nchunks + j + 1) * DD + idx] = nv[q];
      }
      __syncwarp();
    }
  }
}

// ------------------------------------------------------------ backward: carry
// H_{nchunks-1} = 0;  H_{j-1} = P_j^T H_j P_j + c'_j  (one-sided: P_j^T H_j + c'_j)
template <int D, bool TWO>
__global__ void __launch_bounds__(128) bwd_carry_kernel(ScanArgs a) {
  const int64_t S = a.B * a.N;
  if constexpr (D == 4) {
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
  } else {
    constexpr int DD = D * D;
    constexpr int PER = DD / 32;
    __shared__ float sh_h[4][DD];
    __shared__ float sh_P[4][DD];
    __shared__ float sh_y[4][DD];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t s = blockIdx.x * 4 + w;
    if (s >= S) return;
    float* h = sh_h[w];
    float* P = sh_P[w];
    float* y = sh_y[w];
#pragma unroll
    for (int q = 0; q < PER; ++q) {
      const int idx = lane + 32 * q;
      h[idx] = a.hT ? a.hT[s * DD + idx] : 0.0f;
      a.carry[(s * a.nchunks + a.nchunks - 1) * DD + idx] = h[idx];
    }
    __syncwarp();
    float pn[PER], cn[PER];
#pragma unroll
    for (int q = 0; q < PER; ++q) {
      pn[q] = a.aggP[(s * a.nchunks + a.nchunks - 1) * DD + lane + 32 * q];
      cn[q] = a.aggC[(s * a.nchunks + a.nchunks - 1) * DD + lane + 32 * q];
    }
    for (int64_t j = a.nchunks - 1; j >= 1; --j) {
      float cv[PER];
#pragma unroll
      for (int q = 0; q < PER; ++q) {
        P[lane + 32 * q] = pn[q];
        cv[q] = cn[q];
      }
      if (j >= 2) {
#pragma unroll
        for (int q = 0; q < PER; ++q) {
          pn[q] = a.aggP[(s * a.nchunks + j - 1) * DD + lane + 32 * q];
          cn[q] = a.aggC[(s * a.nchunks + j - 1) * DD + lane + 32 * q];
        }
      }
      __syncwarp();
      // y = P^T h
#pragma unroll
      for (int q = 0; q < PER; ++q) {
        const int idx = lane + 32 * q, i = idx / D, jj = idx % D;
        float acc = 0.0f;
#pragma unroll
        for (int k = 0; k < D; ++k) acc = fmaf(P[k * D + i], h[k * D + jj], acc);
        y[idx] = acc;
      }
      __syncwarp();
      float nv[PER];
#pragma unroll
      for (int q = 0; q < PER; ++q) {
        const int idx = lane + 32 * q, i = idx / D, l = idx % D;
        float acc;
        if constexpr (TWO) {  // (P^T h) P
          acc = 0.0f;
#pragma unroll
          for (int k = 0; k < D; ++k) acc = fmaf(y[i * D + k], P[k * D + l], acc);
        } else {
          acc = y[idx];
        }
        nv[q] = acc + cv[q];
      }
      __syncwarp();
#pragma unroll
      for (int q = 0; q < PER; ++q) {
        const int idx = lane + 32 * q;
        h[idx] = nv[q];
        a.carry[(s * a.nchunks + j - 1) * DD + idx] = nv[q];
      }
      __syncwarp();
    }
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

}  // namespace csn
