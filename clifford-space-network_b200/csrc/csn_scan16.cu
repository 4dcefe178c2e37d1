// csn_scan16.cu -- D = 16 (Cl(8,0) ~ M_16(R)) rotor scans.
//
// Same three-phase chunked algorithm as csn_scan.cu (reduce -> carry -> apply, and
// the reverse-time mirror for the adjoint), but a 16 x 16 matrix is too large for
// one thread's registers, so one warp owns one (sequence, chunk).  The warp keeps
// its matrices in shared memory; lane l owns the 8 entries (i, j) with
// j = l % 16 and i = l / 16 + 2q (q = 0..7).
#include "csn_common.cuh"
#include "csn_internal.h"
#include "csn_scan_args.cuh"
#include "csn_carry.cuh"

namespace csn {
namespace s16 {

constexpr int D = 16;
constexpr int DD = 256;
constexpr int WARPS = 4;  // warps per block

// out(i,j) for the lane's 8 entries of A * B (A, B row-major 16 x 16 in smem).
__device__ __forceinline__ void prod_nn(const float* __restrict__ A, const float* __restrict__ B,
                                        float (&o)[8], int lane) {
  const int j = lane & 15, i0 = lane >> 4;
  float bc[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) bc[k] = B[k * 16 + j];
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float4* ar = reinterpret_cast<const float4*>(A + (i0 + 2 * q) * 16);
    float acc = 0.0f;
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const float4 a = ar[v];
      acc = fmaf(a.x, bc[4 * v], acc);
      acc = fmaf(a.y, bc[4 * v + 1], acc);
      acc = fmaf(a.z, bc[4 * v + 2], acc);
      acc = fmaf(a.w, bc[4 * v + 3], acc);
    }
    o[q] = acc;
  }
}

// out = A * B^T
__device__ __forceinline__ void prod_nt(const float* __restrict__ A, const float* __restrict__ B,
                                        float (&o)[8], int lane) {
  const int j = lane & 15, i0 = lane >> 4;
  float bc[16];
  const float4* br = reinterpret_cast<const float4*>(B + j * 16);
#pragma unroll
  for (int v = 0; v < 4; ++v) {
    const float4 b = br[v];
    bc[4 * v] = b.x; bc[4 * v + 1] = b.y; bc[4 * v + 2] = b.z; bc[4 * v + 3] = b.w;
  }
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float4* ar = reinterpret_cast<const float4*>(A + (i0 + 2 * q) * 16);
    float acc = 0.0f;
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const float4 a = ar[v];
      acc = fmaf(a.x, bc[4 * v], acc);
      acc = fmaf(a.y, bc[4 * v + 1], acc);
      acc = fmaf(a.z, bc[4 * v + 2], acc);
      acc = fmaf(a.w, bc[4 * v + 3], acc);
    }
    o[q] = acc;
  }
}

__device__ __forceinline__ int ent(int lane, int q) { return ((lane >> 4) + 2 * q) * 16 + (lane & 15); }
__device__ __forceinline__ int entT(int lane, int q) { return (lane & 15) * 16 + (lane >> 4) + 2 * q; }

__device__ __forceinline__ void put(float* dst, const float (&o)[8], int lane) {
#pragma unroll
  for (int q = 0; q < 8; ++q) dst[ent(lane, q)] = o[q];
}
__device__ __forceinline__ void put2(float* dst, float* dstT, const float (&o)[8], int lane) {
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    dst[ent(lane, q)] = o[q];
    dstT[entT(lane, q)] = o[q];
  }
}
__device__ __forceinline__ void load_lane(float (&o)[8], const float* __restrict__ g, int lane) {
#pragma unroll
  for (int q = 0; q < 8; ++q) o[q] = __ldg(g + ent(lane, q));
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

struct Warp {
  float* M;
  float* Mt;
  float* A;  // state / G
  float* At;
  float* T;
  float* U;
  float* V;
  float* g;  // generators (<= 120)
};

struct BlockTab {
  unsigned char col[CSN_CL8_NBIV][16];
  signed char sgn[CSN_CL8_NBIV][16];
};

// Build M = sa (2 (I - Omega)^{-1} - I) and M^T into w.M / w.Mt.
template <int BASIS, bool DAMPED, int K>
__device__ __forceinline__ void build_M(const ScanArgs& a, const BlockTab& tab, Warp& w, int lane,
                                        int64_t b, int64_t t, int64_t e, float& alpha, float& sa,
                                        float& dtv, float& gam) {
  for (int k = lane; k < K; k += 32) w.g[k] = __ldg(a.gens + e * K + k);
  dtv = __ldg(a.dt + b * a.T + t);
  const float h = 0.5f * dtv;
  __syncwarp();
  float* A = w.T;  // GJ work buffer
  if constexpr (BASIS == BASIS_TRIU) {
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int idx = ent(lane, q), i = idx >> 4, j = idx & 15;
      float v = (i == j) ? 1.0f : 0.0f;
      if (i < j) v = -h * w.g[i * (2 * D - i - 1) / 2 + (j - i - 1)];
      else if (i > j) v = h * w.g[j * (2 * D - j - 1) / 2 + (i - j - 1)];
      A[idx] = v;
    }
  } else {
    if (lane < 16) {
      float row[16];
#pragma unroll
      for (int c = 0; c < 16; ++c) row[c] = (c == lane) ? 1.0f : 0.0f;
      for (int k = 0; k < K; ++k) {
        const float wk = h * w.g[k];
        const int c = tab.col[k][lane];
        const float sg = tab.sgn[k][lane];
#pragma unroll
        for (int cc = 0; cc < 16; ++cc)
          if (cc == c) row[cc] = fmaf(-sg, wk, row[cc]);
      }
#pragma unroll
      for (int c = 0; c < 16; ++c) A[lane * 16 + c] = row[c];
    }
  }
  __syncwarp();
  // Gauss-Jordan inverse in place (pivots >= 1 for I - skew, no pivoting needed)
  for (int k = 0; k < 16; ++k) {
    const float inv = 1.0f / A[k * 16 + k];
    float nv[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int idx = ent(lane, q), i = idx >> 4, j = idx & 15;
      const float aij = A[idx];
      if (i == k && j == k) nv[q] = inv;
      else if (i == k) nv[q] = aij * inv;
      else if (j == k) nv[q] = -aij * inv;
      else nv[q] = aij - A[i * 16 + k] * A[k * 16 + j] * inv;
    }
    __syncwarp();
#pragma unroll
    for (int q = 0; q < 8; ++q) A[ent(lane, q)] = nv[q];
    __syncwarp();
  }
  if constexpr (DAMPED) {
    gam = __ldg(a.gamma + e);
    alpha = 1.0f / (1.0f + expf(gam * dtv));
    sa = sqrtf(alpha);
  } else {
    gam = 0.0f;
    alpha = 1.0f;
    sa = 1.0f;
  }
  float m[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const int idx = ent(lane, q);
    m[q] = sa * (2.0f * A[idx] - (((idx >> 4) == (idx & 15)) ? 1.0f : 0.0f));
  }
  put2(w.M, w.Mt, m, lane);
  __syncwarp();
}

__device__ __forceinline__ void load_tab(BlockTab& tab) {
  constexpr auto t = cl8_biv_tab();
  for (int i = threadIdx.x; i < CSN_CL8_NBIV * 16; i += blockDim.x) {
    tab.col[i / 16][i % 16] = t.col[i / 16][i % 16];
    tab.sgn[i / 16][i % 16] = t.sgn[i / 16][i % 16];
  }
}

#define S16_SETUP()                                                               \
  __shared__ __align__(16) float sm[WARPS][7][DD];                                \
  __shared__ __align__(16) float sg[WARPS][128];                                  \
  __shared__ BlockTab tab;                                                        \
  if (BASIS == BASIS_GA) load_tab(tab);                                           \
  __syncthreads();                                                                \
  const int wi = threadIdx.x >> 5, lane = threadIdx.x & 31;                       \
  const int64_t wid = blockIdx.x * (int64_t)WARPS + wi;                           \
  const int64_t total = a.B * a.N * a.nchunks;                                    \
  if (wid >= total) return;                                                       \
  const int64_t n = wid % a.N;                                                    \
  const int64_t j = (wid / a.N) % a.nchunks;                                      \
  const int64_t b = wid / (a.N * a.nchunks);                                      \
  const int64_t s = b * a.N + n;                                                  \
  const int64_t t0 = j * a.chunk;                                                 \
  const int64_t t1 = min(a.T, t0 + a.chunk);                                      \
  Warp w{sm[wi][0], sm[wi][1], sm[wi][2], sm[wi][3], sm[wi][4], sm[wi][5], sm[wi][6], sg[wi]}; \
  (void)s; (void)t1;

template <int SRC, int BASIS, bool DAMPED, bool TWO>
__global__ void __launch_bounds__(128) fwd_reduce16(ScanArgs a) {
  constexpr int K = GenCount<16, BASIS>::K;
  S16_SETUP();
  // w.A = c (state), w.U = P
  float o[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const int idx = ent(lane, q);
    w.A[idx] = 0.0f;
    w.U[idx] = ((idx >> 4) == (idx & 15)) ? 1.0f : 0.0f;
  }
  __syncwarp();
  for (int64_t t = t0; t < t1; ++t) {
    const int64_t e = (b * a.T + t) * a.N + n;
    float alpha = 1.0f, sa = 1.0f, dtv = 0.0f, gam = 0.0f, cs = 1.0f;
    if constexpr (SRC == SRC_MC) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float v = __ldg(a.M + e * DD + ent(lane, q));
        w.M[ent(lane, q)] = v;
        w.Mt[entT(lane, q)] = v;
      }
      __syncwarp();
    } else {
      build_M<BASIS, DAMPED, K>(a, tab, w, lane, b, t, e, alpha, sa, dtv, gam);
      cs = DAMPED ? (1.0f - alpha) : 1.0f;
    }
    const float* inj = (SRC == SRC_MC) ? (a.C + e * DD) : (a.S + e * DD);
    prod_nn(w.M, w.A, o, lane);  // M c
    __syncwarp();
    if constexpr (TWO) {
      put(w.V, o, lane);
      __syncwarp();
      prod_nt(w.V, w.M, o, lane);  // (M c) M^T
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) o[q] = fmaf(cs, __ldg(inj + ent(lane, q)), o[q]);
    __syncwarp();
    put(w.A, o, lane);
    prod_nn(w.M, w.U, o, lane);  // M P
    __syncwarp();
    put(w.U, o, lane);
    __syncwarp();
  }
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    a.aggP[(s * a.nchunks + j) * DD + ent(lane, q)] = w.U[ent(lane, q)];
    a.aggC[(s * a.nchunks + j) * DD + ent(lane, q)] = w.A[ent(lane, q)];
  }
}

template <int SRC, int BASIS, bool DAMPED, bool TWO>
__global__ void __launch_bounds__(128) fwd_apply16(ScanArgs a) {
  constexpr int K = GenCount<16, BASIS>::K;
  S16_SETUP();
  float o[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const int idx = ent(lane, q);
    float v = 0.0f;
    if (a.nchunks > 1) v = a.carry[(s * a.nchunks + j) * DD + idx];
    else if (a.h0) v = a.h0[s * DD + idx];
    w.A[idx] = v;
  }
  __syncwarp();
  for (int64_t t = t0; t < t1; ++t) {
    const int64_t e = (b * a.T + t) * a.N + n;
    float alpha = 1.0f, sa = 1.0f, dtv = 0.0f, gam = 0.0f, cs = 1.0f;
    if constexpr (SRC == SRC_MC) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float v = __ldg(a.M + e * DD + ent(lane, q));
        w.M[ent(lane, q)] = v;
        w.Mt[entT(lane, q)] = v;
      }
      __syncwarp();
    } else {
      build_M<BASIS, DAMPED, K>(a, tab, w, lane, b, t, e, alpha, sa, dtv, gam);
      cs = DAMPED ? (1.0f - alpha) : 1.0f;
    }
    const float* inj = (SRC == SRC_MC) ? (a.C + e * DD) : (a.S + e * DD);
    prod_nn(w.M, w.A, o, lane);
    __syncwarp();
    if constexpr (TWO) {
      put(w.V, o, lane);
      __syncwarp();
      prod_nt(w.V, w.M, o, lane);
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      o[q] = fmaf(cs, __ldg(inj + ent(lane, q)), o[q]);
      __stcs(a.out + e * DD + ent(lane, q), o[q]);
    }
    __syncwarp();
    put(w.A, o, lane);
    __syncwarp();
  }
}

template <int SRC, int BASIS, bool DAMPED, bool TWO>
__global__ void __launch_bounds__(128) bwd_reduce16(ScanArgs a) {
  constexpr int K = GenCount<16, BASIS>::K;
  S16_SETUP();
  if (j == 0 && !a.agg_mode) return;
  float o[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const int idx = ent(lane, q);
    w.A[idx] = 0.0f;
    w.U[idx] = ((idx >> 4) == (idx & 15)) ? 1.0f : 0.0f;
  }
  __syncwarp();
  for (int64_t t = t1 - 1; t >= t0; --t) {
    const int64_t e = (b * a.T + t) * a.N + n;
    float alpha, sa, dtv, gam;
    if constexpr (SRC == SRC_MC) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float v = __ldg(a.M + e * DD + ent(lane, q));
        w.M[ent(lane, q)] = v;
        w.Mt[entT(lane, q)] = v;
      }
      __syncwarp();
    } else {
      build_M<BASIS, DAMPED, K>(a, tab, w, lane, b, t, e, alpha, sa, dtv, gam);
    }
    // G = g + dX
#pragma unroll
    for (int q = 0; q < 8; ++q) w.A[ent(lane, q)] += __ldg(a.dX + e * DD + ent(lane, q));
    __syncwarp();
    prod_nn(w.Mt, w.A, o, lane);  // M^T G
    __syncwarp();
    if constexpr (TWO) {
      put(w.V, o, lane);
      __syncwarp();
      prod_nn(w.V, w.M, o, lane);  // (M^T G) M
      __syncwarp();
    }
    put(w.A, o, lane);
    prod_nn(w.U, w.M, o, lane);  // P M
    __syncwarp();
    put(w.U, o, lane);
    __syncwarp();
  }
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    a.aggP[(s * a.nchunks + j) * DD + ent(lane, q)] = w.U[ent(lane, q)];
    a.aggC[(s * a.nchunks + j) * DD + ent(lane, q)] = w.A[ent(lane, q)];
  }
}

template <int SRC, int BASIS, bool DAMPED, bool TWO>
__global__ void __launch_bounds__(128) bwd_apply16(ScanArgs a) {
  constexpr int K = GenCount<16, BASIS>::K;
  S16_SETUP();
  float o[8], gq[8];
  // w.A = H (carry from the right), later G;  w.At = G^T
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const int idx = ent(lane, q);
    w.A[idx] = (a.nchunks > 1) ? a.carry[(s * a.nchunks + j) * DD + idx] : a.hT ? a.hT[s * DD + idx] : 0.0f;
  }
  __syncwarp();
  float* Xp = w.U;
  for (int64_t t = t1 - 1; t >= t0; --t) {
    const int64_t e = (b * a.T + t) * a.N + n;
    float alpha = 1.0f, sa = 1.0f, dtv = 0.0f, gam = 0.0f;
    if constexpr (SRC == SRC_MC) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float v = __ldg(a.M + e * DD + ent(lane, q));
        w.M[ent(lane, q)] = v;
        w.Mt[entT(lane, q)] = v;
      }
      __syncwarp();
    } else {
      build_M<BASIS, DAMPED, K>(a, tab, w, lane, b, t, e, alpha, sa, dtv, gam);
    }
    // G = H + dX_t
#pragma unroll
    for (int q = 0; q < 8; ++q) gq[q] = w.A[ent(lane, q)] + __ldg(a.dX + e * DD + ent(lane, q));
    __syncwarp();
    put2(w.A, w.At, gq, lane);
    const float* xprev = (t > 0) ? (a.X + ((b * a.T + t - 1) * a.N + n) * DD)
                                 : (a.h0 ? a.h0 + s * DD : nullptr);
    float dm[8];
    if (xprev) {
#pragma unroll
      for (int q = 0; q < 8; ++q) Xp[ent(lane, q)] = __ldg(xprev + ent(lane, q));
      __syncwarp();
      if constexpr (TWO) {
        prod_nn(w.A, w.M, o, lane);  // G M
        put(w.T, o, lane);
        __syncwarp();
        prod_nt(w.T, Xp, dm, lane);  // G M Xp^T
        prod_nn(w.M, Xp, o, lane);   // M Xp
        __syncwarp();
        put(w.V, o, lane);
        __syncwarp();
        prod_nn(w.At, w.V, o, lane);  // G^T M Xp
#pragma unroll
        for (int q = 0; q < 8; ++q) dm[q] += o[q];
      } else {
        prod_nt(w.A, Xp, dm, lane);  // G Xp^T
      }
    } else {
#pragma unroll
      for (int q = 0; q < 8; ++q) dm[q] = 0.0f;
    }
    __syncwarp();
    if constexpr (SRC == SRC_MC) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        __stcs(a.dM + e * DD + ent(lane, q), dm[q]);
        __stcs(a.dC + e * DD + ent(lane, q), gq[q]);
      }
    } else {
      const float cs = DAMPED ? (1.0f - alpha) : 1.0f;
#pragma unroll
      for (int q = 0; q < 8; ++q) __stcs(a.dC + e * DD + ent(lane, q), cs * gq[q]);
      float da = 0.0f;
      if constexpr (DAMPED) {
        float p1 = 0.0f, p2 = 0.0f;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          p1 = fmaf(dm[q], w.M[ent(lane, q)], p1);
          p2 = fmaf(gq[q], __ldg(a.S + e * DD + ent(lane, q)), p2);
        }
        p1 = warp_sum(p1);
        p2 = warp_sum(p2);
        da = -p2 + p1 / (2.0f * alpha);
      }
      // dQ = sa dM;  V = Bt dQ with Bt = 0.5 (Mt / sa + I);  dOm = 2 V Bt = V (Mt / sa + I)
      const float inv_sa = 1.0f / sa;
#pragma unroll
      for (int q = 0; q < 8; ++q) dm[q] *= sa;
      put(w.T, dm, lane);
      __syncwarp();
      prod_nn(w.Mt, w.T, o, lane);
#pragma unroll
      for (int q = 0; q < 8; ++q) o[q] = 0.5f * (o[q] * inv_sa + dm[q]);
      __syncwarp();
      put(w.V, o, lane);
      __syncwarp();
      float vq[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) vq[q] = o[q];
      prod_nn(w.V, w.Mt, o, lane);
#pragma unroll
      for (int q = 0; q < 8; ++q) o[q] = o[q] * inv_sa + vq[q];
      __syncwarp();
      put(w.T, o, lane);  // dOmega
      __syncwarp();
      float ddt = 0.0f;
      const float hdt = 0.5f * dtv;
      for (int k = lane; k < K; k += 32) {
        float pk;
        if constexpr (BASIS == BASIS_TRIU) {
          // k -> (u, v) in triu order
          int u = 0, rem = k;
          while (rem >= D - 1 - u) { rem -= D - 1 - u; ++u; }
          const int v = u + 1 + rem;
          pk = w.T[u * 16 + v] - w.T[v * 16 + u];
        } else {
          pk = 0.0f;
#pragma unroll
          for (int u = 0; u < 16; ++u) pk = fmaf((float)tab.sgn[k][u], w.T[u * 16 + tab.col[k][u]], pk);
        }
        a.dgens[e * K + k] = pk * hdt;
        ddt = fmaf(pk, 0.5f * w.g[k], ddt);
      }
      ddt = warp_sum(ddt);
      if (lane == 0) {
        if constexpr (DAMPED) {
          const float dz = da * alpha * (1.0f - alpha);
          a.dgamma[e] = -dz * dtv;
          ddt = fmaf(-dz, gam, ddt);
        }
        a.ddt_part[e] = ddt;
      }
    }
    __syncwarp();
    // H <- M^T G M (one-sided M^T G)
    prod_nn(w.Mt, w.A, o, lane);
    __syncwarp();
    if constexpr (TWO) {
      put(w.V, o, lane);
      __syncwarp();
      prod_nn(w.V, w.M, o, lane);
      __syncwarp();
    }
    put(w.A, o, lane);
    __syncwarp();
  }
  if (j == 0 && a.dh0) {
#pragma unroll
    for (int q = 0; q < 8; ++q) a.dh0[s * DD + ent(lane, q)] = w.A[ent(lane, q)];
  }
}

unsigned nblk(int64_t warps) { return (unsigned)((warps + WARPS - 1) / WARPS); }

template <int SRC, int BASIS, bool DAMPED, bool TWO>
int run16(const ScanArgs& a, bool bwd, cudaStream_t st) {
  const int64_t S = a.B * a.N;
  const int64_t total = S * a.nchunks;
  if (a.agg_mode == 1) {
    if (total == 0) return CSN_OK;
    if (!bwd) {
      {
        KernelTimer kt("agg_fwd_reduce", st);
        fwd_reduce16<SRC, BASIS, DAMPED, TWO><<<nblk(total), 128, 0, st>>>(a);
      }
      KernelTimer kt("agg_compose", st);
      compose_kernel<16, TWO, false><<<nblk(S), 128, 0, st>>>(a);
    } else {
      {
        KernelTimer kt("agg_bwd_reduce", st);
        bwd_reduce16<SRC, BASIS, DAMPED, TWO><<<nblk(total), 128, 0, st>>>(a);
      }
      KernelTimer kt("agg_compose", st);
      compose_kernel<16, TWO, true><<<nblk(S), 128, 0, st>>>(a);
    }
    return check_launch("shard aggregate (D=16)");
  }
  if (!bwd) {
    if (total == 0) return CSN_OK;
    if (a.nchunks > 1) {
      if (a.agg_mode != 2) {
        KernelTimer kt("fwd_reduce", st);
        fwd_reduce16<SRC, BASIS, DAMPED, TWO><<<nblk(total), 128, 0, st>>>(a);
      }
      KernelTimer kt("fwd_carry", st);
      launch_grouped_carry<16, TWO, false>(a, st);
    }
    KernelTimer kt("fwd_apply", st);
    fwd_apply16<SRC, BASIS, DAMPED, TWO><<<nblk(total), 128, 0, st>>>(a);
    return check_launch("scan forward (D=16)");
  }
  if (total > 0) {
    if (a.nchunks > 1) {
      if (a.agg_mode != 2) {
        KernelTimer kt("bwd_reduce", st);
        bwd_reduce16<SRC, BASIS, DAMPED, TWO><<<nblk(total), 128, 0, st>>>(a);
      }
      KernelTimer kt("bwd_carry", st);
      launch_grouped_carry<16, TWO, true>(a, st);
    }
    KernelTimer kt("bwd_apply", st);
    bwd_apply16<SRC, BASIS, DAMPED, TWO><<<nblk(total), 128, 0, st>>>(a);
  }
  if (SRC == SRC_ROTOR && a.B * a.T > 0) {
    const int64_t BT = a.B * a.T;
    KernelTimer kt("reduce_channels", st);
    reduce_channels_kernel<<<(unsigned)((BT + 255) / 256), 256, 0, st>>>(a.ddt_part, a.ddt, BT, a.N);
  }
  return check_launch("scan backward (D=16)");
}

template <int SRC, int BASIS, bool DAMPED>
int run16s(const ScanArgs& a, bool two, bool bwd, cudaStream_t st) {
  return two ? run16<SRC, BASIS, DAMPED, true>(a, bwd, st) : run16<SRC, BASIS, DAMPED, false>(a, bwd, st);
}

}  // namespace s16

int scan16_dispatch(const ScanArgs& a, int src, int basis, bool damped, bool two, bool bwd,
                    cudaStream_t st) {
  using namespace s16;
  if (src == SRC_MC) return run16s<SRC_MC, BASIS_TRIU, false>(a, two, bwd, st);
  if (basis == BASIS_TRIU)
    return damped ? run16s<SRC_ROTOR, BASIS_TRIU, true>(a, two, bwd, st)
                  : run16s<SRC_ROTOR, BASIS_TRIU, false>(a, two, bwd, st);
  return damped ? run16s<SRC_ROTOR, BASIS_GA, true>(a, two, bwd, st)
                : run16s<SRC_ROTOR, BASIS_GA, false>(a, two, bwd, st);
}

}  // namespace csn
