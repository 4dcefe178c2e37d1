// csn_scan.cu -- chunked rotor scans for sm_100a (D = 4, 8).
//
// Recurrence (per sequence s = (b, n), X_{-1} = h0 or 0):
//   two-sided  X_t = M_t X_{t-1} M_t^T + C_t     (python/clifford_scan.py:19-85)
//   one-sided  X_t = M_t X_{t-1} + C_t           (csn_toolkit/csn/scan.py:16-41)
// with (M_t, C_t) either given (plain scan) or built on the fly from generators,
// dt, gamma and S (fused rotor scan, python/clifford_cl6.py:150-171):
//   Omega = 0.5 dt sum_k g_k E_k, Q = (I - Omega)^{-1}(I + Omega) = 2 (I - Omega)^{-1} - I,
//   damped:   a = sigmoid(-gamma dt), M = sqrt(a) Q, C = (1 - a) S
//   undamped: M = Q, C = S.
//
// Parallel structure (work-efficient reduce-then-scan over time chunks; one thread
// owns one (sequence, chunk) and keeps its D x D matrices in registers):
//   1. reduce: each chunk j computes its aggregate (P_j, c_j): P_j = M_end ... M_start,
//      c_j = chunk-local scan result with zero carry-in;
//   2. carry:  per sequence, h_{j+1} = P_j h_j P_j^T + c_j (one-sided: P_j h_j + c_j),
//      h_0 = h0;
//   3. apply:  each chunk rescans from its carry h_j and writes X.
// The backward pass is the mirror image in reverse time with transitions M^T
// (G_t = dX_t + M_{t+1}^T G_{t+1} M_{t+1}), chunk aggregates (P_j, c'_j) where
// H_{j-1} = P_j^T H_j P_j + c'_j, and an apply pass that emits the gradients.
#include <algorithm>
#include <climits>
#include <cstdio>
#include <mutex>

#include "csn_common.cuh"
#include "csn_internal.h"
#include "csn_scan_args.cuh"
#include "csn_carry.cuh"

namespace csn {

// Build M_t of the fused rotor scan.  Writes M and the rotor scalars.
template <int D, int BASIS, bool DAMPED, int K>
__device__ __forceinline__ void rotor_transition(const ScanArgs& a, int64_t b, int64_t t,
                                                 int64_t e, Mat<D>& M, RotorStep<D, K>& r) {
  load_gens<K>(r.g, a.gens + e * K);
  const int64_t tp = tphys(a, t);
  r.dt = __ldg(a.dt + dt_index(a, b, tp, e - (b * a.T + tp) * a.N));
  build_neg_omega<D, BASIS, K>(M, r.g, 0.5f * r.dt);
  gj_inverse_dev(M);  // M = A^{-1} - I
  if constexpr (DAMPED) {
    r.gamma = __ldg(a.gamma + e);
    r.alpha = 1.0f / (1.0f + expf(r.gamma * r.dt));
    r.sa = sqrtf(r.alpha);
  } else {
    r.gamma = 0.0f;
    r.alpha = 1.0f;
    r.sa = 1.0f;
  }
  rotor_from_dev(M, r.sa);  // M = sa (2 A^{-1} - I)
}

// Load/build the transition M_t; returns the scale applied to the injected matrix
// (C_t = cscale * S_t for the rotor source, C_t itself for the plain source).
template <int D, int SRC, int BASIS, bool DAMPED, int K>
__device__ __forceinline__ float transition(const ScanArgs& a, int64_t b, int64_t t, int64_t e,
                                            Mat<D>& M, RotorStep<D, K>& r) {
  if constexpr (SRC == SRC_MC) {
    load_mat(M, a.M + e * (D * D));
    return 1.0f;
  } else {
    rotor_transition<D, BASIS, DAMPED, K>(a, b, t, e, M, r);
    return DAMPED ? (1.0f - r.alpha) : 1.0f;
  }
}

template <int D, int SRC>
__device__ __forceinline__ const float* injected(const ScanArgs& a, int64_t e) {
  return (SRC == SRC_MC) ? (a.C + e * (D * D)) : (a.S + e * (D * D));
}

// ------------------------------------------------------------ forward: reduce
template <int D, int SRC, int BASIS, bool DAMPED, bool TWO>
__global__ void __launch_bounds__(128) fwd_reduce_kernel(ScanArgs a) {
  constexpr int K = GenCount<D, BASIS>::K;
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t total = a.B * a.N * a.nchunks;
  if (tid >= total) return;
  const int64_t n = tid % a.N;
  const int64_t j = (tid / a.N) % a.nchunks;
  const int64_t b = tid / (a.N * a.nchunks);
  const int64_t t0 = j * a.chunk;
  const int64_t t1 = min(a.T, t0 + a.chunk);

  Mat<D> P, c, M;
  mat_identity(P);
  mat_zero(c);
  RotorStep<D, K> r;
  for (int64_t t = t0; t < t1; ++t) {
    const int64_t e = elem(a, b, t, n);
    const float cs = transition<D, SRC, BASIS, DAMPED, K>(a, b, t, e, M, r);
    lmul(M, c);
    if constexpr (TWO) rmulT(c, M);
    add_scaled_mat(c, injected<D, SRC>(a, e), cs);
    lmul(M, P);
  }
  const int64_t s = b * a.N + n;
  store_mat(a.aggP + (s * a.nchunks + j) * (D * D), P);
  store_mat(a.aggC + (s * a.nchunks + j) * (D * D), c);
}

// ------------------------------------------------------------ forward: apply
template <int D, int SRC, int BASIS, bool DAMPED, bool TWO>
__global__ void __launch_bounds__(128) fwd_apply_kernel(ScanArgs a) {
  constexpr int K = GenCount<D, BASIS>::K;
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t total = a.B * a.N * a.nchunks;
  if (tid >= total) return;
  const int64_t n = tid % a.N;
  const int64_t j = (tid / a.N) % a.nchunks;
  const int64_t b = tid / (a.N * a.nchunks);
  const int64_t s = b * a.N + n;
  const int64_t t0 = j * a.chunk;
  const int64_t t1 = min(a.T, t0 + a.chunk);

  Mat<D> X, M;
  if (a.nchunks > 1) load_mat(X, a.carry + (s * a.nchunks + j) * (D * D));
  else if (a.h0) load_mat(X, a.h0 + s * (D * D));
  else mat_zero(X);
  RotorStep<D, K> r;
  for (int64_t t = t0; t < t1; ++t) {
    const int64_t e = elem(a, b, t, n);
    const float cs = transition<D, SRC, BASIS, DAMPED, K>(a, b, t, e, M, r);
    lmul(M, X);
    if constexpr (TWO) rmulT(X, M);
    add_scaled_mat(X, injected<D, SRC>(a, e), cs);
    store_mat_cs(a.out + e * (D * D), X);
  }
}

// ------------------------------------------------------------ backward: reduce
// Chunk aggregate of the reverse recurrence with zero carry from the right:
//   g <- 0; for t = end..start: G = dX_t + g; g = M_t^T G M_t (one-sided M_t^T G)
//   P = M_end ... M_start.
template <int D, int SRC, int BASIS, bool DAMPED, bool TWO>
__global__ void __launch_bounds__(128) bwd_reduce_kernel(ScanArgs a) {
  constexpr int K = GenCount<D, BASIS>::K;
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t total = a.B * a.N * a.nchunks;
  if (tid >= total) return;
  const int64_t n = tid % a.N;
  const int64_t j = (tid / a.N) % a.nchunks;
  const int64_t b = tid / (a.N * a.nchunks);
  if (j == 0 && !a.agg_mode) return;  // chunk 0's aggregate only matters for shard aggregates
  const int64_t t0 = j * a.chunk;
  const int64_t t1 = min(a.T, t0 + a.chunk);

  Mat<D> P, g, M;
  mat_identity(P);
  mat_zero(g);
  RotorStep<D, K> r;
  for (int64_t t = t1 - 1; t >= t0; --t) {
    const int64_t e = elem(a, b, t, n);
    transition<D, SRC, BASIS, DAMPED, K>(a, b, t, e, M, r);
    add_scaled_mat(g, a.dX + e * (D * D), 1.0f);
    lmulT(M, g);
    if constexpr (TWO) rmul(g, M);
    if (!a.reuse_P) rmul(P, M);
  }
  const int64_t s = b * a.N + n;
  if (!a.reuse_P) store_mat(a.aggP + (s * a.nchunks + j) * (D * D), P);
  store_mat(a.aggC + (s * a.nchunks + j) * (D * D), g);
}

// ------------------------------------------------------------ backward: apply
template <int D, int SRC, int BASIS, bool DAMPED, bool TWO>
__global__ void __launch_bounds__(128) bwd_apply_kernel(ScanArgs a) {
  constexpr int K = GenCount<D, BASIS>::K;
  constexpr int DD = D * D;
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t total = a.B * a.N * a.nchunks;
  if (tid >= total) return;
  const int64_t n = tid % a.N;
  const int64_t j = (tid / a.N) % a.nchunks;
  const int64_t b = tid / (a.N * a.nchunks);
  const int64_t s = b * a.N + n;
  const int64_t t0 = j * a.chunk;
  const int64_t t1 = min(a.T, t0 + a.chunk);

  Mat<D> H, M;
  if (a.nchunks > 1) load_mat(H, a.carry + (s * a.nchunks + j) * DD);
  else if (a.hT) load_mat(H, a.hT + s * DD);
  else mat_zero(H);
  RotorStep<D, K> r;
  for (int64_t t = t1 - 1; t >= t0; --t) {
    const int64_t e = elem(a, b, t, n);
    transition<D, SRC, BASIS, DAMPED, K>(a, b, t, e, M, r);
    // G = dX_t + H (held in H)
    add_scaled_mat(H, a.dX + e * DD, 1.0f);
    const float* xprev = (t > 0) ? (a.X + elem(a, b, t - 1, n) * DD) : a.h0 ? (a.h0 + s * DD) : nullptr;

    // dM = G M Xp^T + G^T M Xp (two-sided) | G Xp^T (one-sided)
    Mat<D> dM;
    if (xprev) {
      Mat<D> Xp;
      load_mat(Xp, xprev);
      if constexpr (TWO) {
        Mat<D> W = H;
        rmul(W, M);    // G M
        rmulT(W, Xp);  // G M Xp^T
        lmul(M, Xp);   // M Xp
        // dM = W + G^T (M Xp)
#pragma unroll
        for (int jj = 0; jj < D; ++jj)
#pragma unroll
          for (int i = 0; i < D; ++i) {
            float acc = W.a[i][jj];
#pragma unroll
            for (int k = 0; k < D; ++k) acc = fmaf(H.a[k][i], Xp.a[k][jj], acc);
            dM.a[i][jj] = acc;
          }
      } else {
        dM = H;
        rmulT(dM, Xp);
      }
    } else {
      mat_zero(dM);
    }

    if constexpr (SRC == SRC_MC) {
      store_mat_cs(a.dM + e * DD, dM);
      store_mat_cs(a.dC + e * DD, H);
    } else {
      // dS = (1 - a) G  (undamped: G)
      const float cs = DAMPED ? (1.0f - r.alpha) : 1.0f;
      {
        Mat<D> dS;
#pragma unroll
        for (int i = 0; i < D; ++i)
#pragma unroll
          for (int jj = 0; jj < D; ++jj) dS.a[i][jj] = cs * H.a[i][jj];
        store_mat_cs(a.dC + e * DD, dS);
      }
      float da = 0.0f;
      if constexpr (DAMPED) {
        // da = -<G, S> + <dM, M> / (2 a)
        float dmm = 0.0f;
#pragma unroll
        for (int i = 0; i < D; ++i)
#pragma unroll
          for (int jj = 0; jj < D; ++jj) dmm = fmaf(dM.a[i][jj], M.a[i][jj], dmm);
        da = -mat_dot_global(H, a.S + e * DD) + dmm / (2.0f * r.alpha);
      }
      // dQ = sa dM;  dOm = 2 Bt dQ Bt with Bt = A^{-T} = 0.5 (Q^T + I), Q = M / sa
      const float inv_sa = 1.0f / r.sa;
      Mat<D> Bt;
#pragma unroll
      for (int i = 0; i < D; ++i)
#pragma unroll
        for (int jj = 0; jj < D; ++jj)
          Bt.a[i][jj] = 0.5f * (M.a[jj][i] * inv_sa + ((i == jj) ? 1.0f : 0.0f));
#pragma unroll
      for (int i = 0; i < D; ++i)
#pragma unroll
        for (int jj = 0; jj < D; ++jj) dM.a[i][jj] *= 2.0f * r.sa;
      lmul(Bt, dM);  // Bt dQ
      rmul(dM, Bt);  // Bt dQ Bt
      float proj[K];
      project_generators<D, BASIS, K>(dM, proj);
      const float hdt = 0.5f * r.dt;
      float ddt = 0.0f;
      float outg[K];
#pragma unroll
      for (int k = 0; k < K; ++k) {
        outg[k] = proj[k] * hdt;
        ddt = fmaf(proj[k], 0.5f * r.g[k], ddt);
      }
      float* dg = a.dgens + e * K;
      if constexpr (K % 4 == 0) {
#pragma unroll
        for (int v = 0; v < K / 4; ++v)
          __stcs(reinterpret_cast<float4*>(dg) + v,
                 make_float4(outg[4 * v], outg[4 * v + 1], outg[4 * v + 2], outg[4 * v + 3]));
      } else {
#pragma unroll
        for (int k = 0; k < K; ++k) dg[k] = outg[k];
      }
      if constexpr (DAMPED) {
        const float dz = da * r.alpha * (1.0f - r.alpha);
        a.dgamma[e] = -dz * r.dt;
        ddt = fmaf(-dz, r.gamma, ddt);
      }
      a.ddt_part[e] = ddt;
    }
    // H <- M^T G M (one-sided: M^T G)
    lmulT(M, H);
    if constexpr (TWO) rmul(H, M);
  }
  if (j == 0 && a.dh0) store_mat(a.dh0 + s * DD, H);
}

// ================================================================= host side
// Implemented in csn_scan16.cu (D = 16 kernel family).
int scan16_dispatch(const ScanArgs& a, int src, int basis, bool damped, bool two, bool bwd,
                    cudaStream_t st);
// Implemented in csn_scan8.cu (staged D = 8 fused rotor kernels).
int scan8_rotor_dispatch(const ScanArgs& a, bool damped, bool two, bool bwd, cudaStream_t st);
int scan8_rotor_step(const float* gens, const float* dt, const float* gamma, const float* S, float* h,
                     int64_t B, int64_t N, bool two, bool chained, cudaStream_t st);

namespace {

// D = 16 (one warp per chunk): the rotor-building reduce and the backward apply hold 12 warps
// per SM (registers), so a pass over S sequences cut into n chunks takes about
// ceil(S n / (148 * 12)) waves of one chunk each; more than one chunk adds the reduce pass
// (about as long as the apply pass) and the carry.  The chunk count minimises
//   waves(n) * (chunk(n) + 4) * (n > 1 ? 2 : 1) + (n > 1 ? 32 : 0)
// (4 steps' worth of per-chunk set-up, 32 for the extra launches): long sequences get
// enough chunks that the last wave's tail idles the SMs for a small part of a pass (B16
// L8192 C32: 38 chunks; 5 chunks took 23.7 ms per step, 24 - 64 chunks 19.3 - 19.6 ms),
// while many short sequences that already fill the SMs stay in one chunk (no reduce pass).
static int64_t pick_chunk16(int64_t S, int64_t T) {
  const int64_t slots = 148 * 12;
  const int64_t n_max = std::max<int64_t>(1, std::min<int64_t>(T / 8, (16 * slots + S - 1) / std::max<int64_t>(S, 1)));
  int64_t best_chunk = T, best_cost = -1;
  for (int64_t n = 1; n <= n_max; ++n) {
    const int64_t chunk = std::max<int64_t>(8, (T + n - 1) / n);
    const int64_t nn = (T + chunk - 1) / chunk;
    const int64_t waves = (S * nn + slots - 1) / slots;
    const int64_t cost = waves * (chunk + 4) * (nn > 1 ? 2 : 1) + (nn > 1 ? 32 : 0);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best_chunk = chunk;
    }
  }
  return std::min<int64_t>(best_chunk, T);
}

int64_t pick_chunk(int64_t S, int64_t T, int D) {
  if (D == 16) return T > 0 ? pick_chunk16(S, T) : 1;
  // Enough (sequence, chunk) work items to fill 148 SMs at the residency each family
  // allows: D = 4 ~1024 threads / SM, D = 8 ~256 threads / SM (register bound, one wave).
  // A problem of at most 1024 elements cannot fill the GPU either way and is bound by its
  // launches: one chunk per sequence runs the apply pass alone, without the reduce and
  // carry passes (the reference's D = 4 benchmark, B2 T80: 0.37 -> 0.23 ms per fwd + bwd step).
  if (S * T <= 1024) return T > 0 ? T : 1;
  const int64_t target = (D == 8) ? 148 * 256 : 148 * 1024;
  int64_t chunk = (S * T + target - 1) / target;
  if (chunk < 8) chunk = 8;
  if (chunk > T) chunk = T > 0 ? T : 1;
  return chunk;
}

struct Plan {
  int64_t nchunks, chunk;
  size_t agg_floats;   // aggP + aggC + carry
  size_t part_floats;  // ddt partials (rotor backward)
};

Plan make_plan(int64_t B, int64_t T, int64_t N, int D, bool rotor_bwd) {
  Plan p;
  const int64_t S = B * N;
  p.chunk = pick_chunk(S, T, D);
  p.nchunks = T > 0 ? (T + p.chunk - 1) / p.chunk : 0;
  p.agg_floats = p.nchunks > 1 ? (size_t)3 * S * p.nchunks * D * D : 0;
  p.part_floats = rotor_bwd ? (size_t)B * T * N : 0;
  return p;
}

size_t plan_bytes(const Plan& p) { return (p.agg_floats + p.part_floats) * sizeof(float) + 256; }

struct Workspace {
  float* base = nullptr;
  bool owned = false;
  cudaStream_t stream = nullptr;
  ~Workspace() {
    if (owned && base) cudaFreeAsync(base, stream);
  }
};

int get_ws(Workspace& w, void* user, size_t user_bytes, size_t need, cudaStream_t st) {
  w.stream = st;
  if (need <= 256) return CSN_OK;  // single-chunk plan: no scratch at all
  if (user) {
    if (user_bytes < need) return set_error(CSN_ERR_INVALID, "workspace smaller than *_workspace_bytes()");
    w.base = static_cast<float*>(user);
    return CSN_OK;
  }
  cudaError_t e = cudaMallocAsync(reinterpret_cast<void**>(&w.base), need, st);
  if (e != cudaSuccess) return set_cuda_error(e, "cudaMallocAsync(workspace)");
  w.owned = true;
  return CSN_OK;
}

void bind_ws(ScanArgs& a, const Plan& p, float* base, int D) {
  const int64_t S = a.B * a.N;
  const size_t one = (size_t)S * p.nchunks * D * D;
  float* aligned = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(base) + 255) & ~uintptr_t(255));
  a.aggP = aligned;
  a.aggC = aligned + one;
  a.carry = aligned + 2 * one;
  a.ddt_part = aligned + p.agg_floats;
  a.nchunks = p.nchunks;
  a.chunk = p.chunk;
}

unsigned blocks_for(int64_t n, int threads) { return (unsigned)((n + threads - 1) / threads); }

template <int D, int SRC, int BASIS, bool DAMPED, bool TWO>
int run_fwd(ScanArgs a, cudaStream_t st) {
  const int64_t S = a.B * a.N;
  const int64_t total = S * a.nchunks;
  if (total == 0) return CSN_OK;
  if (a.agg_mode == 1) {
    {
      KernelTimer kt("agg_fwd_reduce", st);
      fwd_reduce_kernel<D, SRC, BASIS, DAMPED, TWO><<<blocks_for(total, 128), 128, 0, st>>>(a);
    }
    KernelTimer kt("agg_compose", st);
    compose_kernel<D, TWO, false><<<blocks_for(S, 4), 128, 0, st>>>(a);
    return check_launch("shard aggregate (forward)");
  }
  if (a.nchunks > 1) {
    if (a.agg_mode != 2) {
      KernelTimer kt("fwd_reduce", st);
      fwd_reduce_kernel<D, SRC, BASIS, DAMPED, TWO><<<blocks_for(total, 128), 128, 0, st>>>(a);
    }
    KernelTimer kt("fwd_carry", st);
    if constexpr (D == 4) fwd_carry_kernel<D, TWO><<<blocks_for(S, 128), 128, 0, st>>>(a);
    else launch_grouped_carry<D, TWO, false>(a, st);
  }
  {
    KernelTimer kt("fwd_apply", st);
    fwd_apply_kernel<D, SRC, BASIS, DAMPED, TWO><<<blocks_for(total, 128), 128, 0, st>>>(a);
  }
  return check_launch("scan forward");
}

template <int D, int SRC, int BASIS, bool DAMPED, bool TWO>
int run_bwd(ScanArgs a, cudaStream_t st) {
  const int64_t S = a.B * a.N;
  const int64_t total = S * a.nchunks;
  if (a.agg_mode == 1) {
    if (total == 0) return CSN_OK;
    {
      KernelTimer kt("agg_bwd_reduce", st);
      bwd_reduce_kernel<D, SRC, BASIS, DAMPED, TWO><<<blocks_for(total, 128), 128, 0, st>>>(a);
    }
    KernelTimer kt("agg_compose", st);
    compose_kernel<D, TWO, true><<<blocks_for(S, 4), 128, 0, st>>>(a);
    return check_launch("shard aggregate (backward)");
  }
  if (total > 0) {
    if (a.nchunks > 1) {
      if (a.agg_mode != 2) {
        KernelTimer kt("bwd_reduce", st);
        bwd_reduce_kernel<D, SRC, BASIS, DAMPED, TWO><<<blocks_for(total, 128), 128, 0, st>>>(a);
      }
      KernelTimer kt("bwd_carry", st);
      if constexpr (D == 4) bwd_carry_kernel<D, TWO><<<blocks_for(S, 128), 128, 0, st>>>(a);
      else launch_grouped_carry<D, TWO, true>(a, st);
    }
    KernelTimer kt("bwd_apply", st);
    bwd_apply_kernel<D, SRC, BASIS, DAMPED, TWO><<<blocks_for(total, 128), 128, 0, st>>>(a);
  }
  if (SRC == SRC_ROTOR && a.B * a.T > 0) {
    const int64_t BT = a.B * a.T;
    KernelTimer kt("reduce_channels", st);
    const int64_t H = dt_heads(a);
    reduce_channels_kernel<<<blocks_for(BT * H, 256), 256, 0, st>>>(a.ddt_part, a.ddt, BT * H, a.N / H);
  }
  return check_launch("scan backward");
}

template <int D, int SRC, int BASIS, bool DAMPED>
int run_sided(ScanArgs a, bool two, bool bwd, cudaStream_t st) {
  if (bwd) return two ? run_bwd<D, SRC, BASIS, DAMPED, true>(a, st) : run_bwd<D, SRC, BASIS, DAMPED, false>(a, st);
  return two ? run_fwd<D, SRC, BASIS, DAMPED, true>(a, st) : run_fwd<D, SRC, BASIS, DAMPED, false>(a, st);
}

int dispatch(ScanArgs a, int D, int src, int basis, bool damped, bool two, bool bwd, cudaStream_t st) {
  if (src == SRC_MC) {
    switch (D) {
      case 4: return run_sided<4, SRC_MC, BASIS_TRIU, false>(a, two, bwd, st);
      case 8: return run_sided<8, SRC_MC, BASIS_TRIU, false>(a, two, bwd, st);
      default: break;
    }
    return set_error(CSN_ERR_UNSUPPORTED, "plain scan: D must be 4 or 8 in this kernel family");
  }
  if (D == 4 && basis == BASIS_TRIU)
    return damped ? run_sided<4, SRC_ROTOR, BASIS_TRIU, true>(a, two, bwd, st)
                  : run_sided<4, SRC_ROTOR, BASIS_TRIU, false>(a, two, bwd, st);
  if (D == 4 && basis == BASIS_GA)
    return damped ? run_sided<4, SRC_ROTOR, BASIS_GA, true>(a, two, bwd, st)
                  : run_sided<4, SRC_ROTOR, BASIS_GA, false>(a, two, bwd, st);
  if (D == 8 && basis == BASIS_TRIU) return scan8_rotor_dispatch(a, damped, two, bwd, st);
  return set_error(CSN_ERR_UNSUPPORTED, "rotor scan: unsupported (D, basis) for this kernel family");
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool aligned8(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7u) == 0; }

int check_shape(int64_t B, int64_t T, int64_t N, int D) {
  if (B < 0 || T < 0 || N < 0) return set_error(CSN_ERR_INVALID, "negative dimension");
  if (D != 4 && D != 8 && D != 16) return set_error(CSN_ERR_INVALID, "D must be 4, 8 or 16");
  return CSN_OK;
}

}  // namespace


}  // namespace csn

using namespace csn;

extern "C" size_t csn_scan_workspace_bytes(int64_t B, int64_t T, int64_t N, int D) {
  if (B < 0 || T < 0 || N < 0 || D < 1) return 0;
  return plan_bytes(make_plan(B, T, N, D, false));
}

extern "C" size_t csn_rotor_scan_workspace_bytes(int64_t B, int64_t T, int64_t N, int D) {
  if (B < 0 || T < 0 || N < 0 || D < 1) return 0;
  return plan_bytes(make_plan(B, T, N, D, true));
}

extern "C" int csn_scan_fwd(const float* M, const float* C, const float* h0, float* X, int64_t B,
                            int64_t T, int64_t N, int D, int flags, void* workspace,
                            size_t workspace_bytes, void* stream) {
  if (int rc = check_shape(B, T, N, D)) return rc;
  if (flags & ~(CSN_SCAN_TWO_SIDED | CSN_SCAN_REVERSE)) return set_error(CSN_ERR_INVALID, "csn_scan_fwd: unknown flags");
  if (B * T * N == 0) return CSN_OK;
  if (!M || !C || !X) return set_error(CSN_ERR_INVALID, "csn_scan_fwd: M, C and X are required");
  if (!aligned16(M) || !aligned16(C) || !aligned16(X) || (h0 && !aligned16(h0)))
    return set_error(CSN_ERR_INVALID, "csn_scan_fwd: pointers must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Plan p = make_plan(B, T, N, D, false);
  Workspace ws;
  if (int rc = get_ws(ws, workspace, workspace_bytes, plan_bytes(p), st)) return rc;
  ScanArgs a{};
  a.M = M; a.C = C; a.h0 = h0; a.out = X; a.B = B; a.T = T; a.N = N;
  a.rev = (flags & CSN_SCAN_REVERSE) != 0;
  const bool two = (flags & CSN_SCAN_TWO_SIDED) != 0;
  bind_ws(a, p, ws.base, D);
  if (D == 16) return scan16_dispatch(a, SRC_MC, BASIS_TRIU, false, two, false, st);
  return dispatch(a, D, SRC_MC, BASIS_TRIU, false, two, false, st);
}

extern "C" int csn_scan_bwd(const float* M, const float* X, const float* dX, const float* h0,
                            float* dM, float* dC, float* dh0, int64_t B, int64_t T, int64_t N,
                            int D, int flags, void* workspace, size_t workspace_bytes,
                            void* stream) {
  if (int rc = check_shape(B, T, N, D)) return rc;
  if (flags & ~(CSN_SCAN_TWO_SIDED | CSN_SCAN_REVERSE)) return set_error(CSN_ERR_INVALID, "csn_scan_bwd: unknown flags");
  if (B * T * N == 0) return CSN_OK;
  if (!M || !X || !dX || !dM || !dC)
    return set_error(CSN_ERR_INVALID, "csn_scan_bwd: M, X, dX, dM and dC are required");
  if (!aligned16(M) || !aligned16(X) || !aligned16(dX) || !aligned16(dM) || !aligned16(dC) ||
      (h0 && !aligned16(h0)) || (dh0 && !aligned16(dh0)))
    return set_error(CSN_ERR_INVALID, "csn_scan_bwd: pointers must be 16-byte aligned");
  if (dh0 && !h0) return set_error(CSN_ERR_INVALID, "csn_scan_bwd: dh0 needs h0");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Plan p = make_plan(B, T, N, D, false);
  Workspace ws;
  if (int rc = get_ws(ws, workspace, workspace_bytes, plan_bytes(p), st)) return rc;
  ScanArgs a{};
  a.M = M; a.X = X; a.dX = dX; a.h0 = h0; a.dM = dM; a.dC = dC; a.dh0 = dh0;
  a.B = B; a.T = T; a.N = N;
  a.rev = (flags & CSN_SCAN_REVERSE) != 0;
  const bool two = (flags & CSN_SCAN_TWO_SIDED) != 0;
  bind_ws(a, p, ws.base, D);
  if (D == 16) return scan16_dispatch(a, SRC_MC, BASIS_TRIU, false, two, true, st);
  return dispatch(a, D, SRC_MC, BASIS_TRIU, false, two, true, st);
}

static int rotor_common_checks(const float* gens, const float* dt, const float* S, int64_t B,
                               int64_t T, int64_t N, int D, int basis) {
  if (int rc = check_shape(B, T, N, D)) return rc;
  if (basis != BASIS_TRIU && basis != BASIS_GA) return set_error(CSN_ERR_INVALID, "unknown basis");
  if (basis == BASIS_GA && D == 8)
    return set_error(CSN_ERR_UNSUPPORTED, "GA basis is provided for D = 4 (Cl(3,0)) and D = 16 (Cl(8,0))");
  if (B * T * N == 0) return CSN_OK;
  if (!gens || !dt || !S) return set_error(CSN_ERR_INVALID, "rotor scan: gens, dt and S are required");
  const int K = (basis == BASIS_GA) ? (D == 4 ? CSN_CL3_NBIV : CSN_CL8_NBIV) : D * (D - 1) / 2;
  if (K % 4 == 0 ? !aligned16(gens) : !aligned8(gens))
    return set_error(CSN_ERR_INVALID, "rotor scan: gens misaligned");
  if (!aligned16(S)) return set_error(CSN_ERR_INVALID, "rotor scan: S must be 16-byte aligned");
  return CSN_OK;
}

namespace {

int fail(int code, const char* fn, const char* what) {
  char buf[320];
  snprintf(buf, sizeof(buf), "%s: %s", fn, what);
  return set_error(code, buf);
}

// H heads: the N channels are H groups of N / H neurons and dt holds one value per head,
// [B, T, H] (H = 1: [B, T]); ddt has the shape of dt.
int check_heads(const char* fn, int64_t N, int64_t H) {
  if (H < 0 || (H == 0 && N != 0)) return fail(CSN_ERR_INVALID, fn, "the head count must be >= 1");
  if (H > 1 && (N % H != 0 || N > INT32_MAX))
    return fail(CSN_ERR_INVALID, fn, "channels must split evenly into heads (N = H * Nh < 2^31)");
  return CSN_OK;
}

int zero_ddt(float* ddt, int64_t n, cudaStream_t st) {
  if (n <= 0 || !ddt) return CSN_OK;
  cudaError_t e = cudaMemsetAsync(ddt, 0, sizeof(float) * n, st);
  return e == cudaSuccess ? CSN_OK : set_cuda_error(e, "cudaMemsetAsync(ddt)");
}

// Forward of every fused-rotor entry point.  Mc_out (D = 16 only): also store each step's M_t.
int rotor_fwd_impl(const char* fn, const float* gens, const float* dt, const float* gamma,
                   const float* S, const float* h0, float* X, float* Mc_out, int64_t B, int64_t T,
                   int64_t N, int64_t H, int D, int basis, int two_sided, void* workspace,
                   size_t workspace_bytes, cudaStream_t st) {
  if (int rc = rotor_common_checks(gens, dt, S, B, T, N, D, basis)) return rc;
  if (int rc = check_heads(fn, N, H)) return rc;
  if (Mc_out && D != 16) return fail(CSN_ERR_UNSUPPORTED, fn, "the rotor cache is for D = 16");
  if (B * T * N == 0) return CSN_OK;
  if (!X || !aligned16(X) || (h0 && !aligned16(h0)) || (Mc_out && !aligned16(Mc_out)))
    return fail(CSN_ERR_INVALID, fn, "X missing or X, h0, Mcache misaligned");
  Plan p = make_plan(B, T, N, D, false);
  Workspace ws;
  if (int rc = get_ws(ws, workspace, workspace_bytes, plan_bytes(p), st)) return rc;
  ScanArgs a{};
  a.gens = gens; a.dt = dt; a.gamma = gamma; a.S = S; a.h0 = h0; a.out = X;
  a.B = B; a.T = T; a.N = N;
  a.dtH = H;
  a.Mc_out = Mc_out;
  bind_ws(a, p, ws.base, D);
  if (D == 16) return scan16_dispatch(a, SRC_ROTOR, basis, gamma != nullptr, two_sided != 0, false, st);
  return dispatch(a, D, SRC_ROTOR, basis, gamma != nullptr, two_sided != 0, false, st);
}

// Adjoint of every fused-rotor entry point.  Mc_in (D = 16 only): the forward's stored
// rotors; reuse: the workspace is the forward's, whose chunk products P_j are reused.
int rotor_bwd_impl(const char* fn, const float* gens, const float* dt, const float* gamma,
                   const float* S, const float* h0, const float* X, const float* dX,
                   const float* Mc_in, float* dgens, float* ddt, float* dgamma, float* dS, float* dh0,
                   int64_t B, int64_t T, int64_t N, int64_t H, int D, int basis, int two_sided,
                   bool reuse, void* workspace, size_t workspace_bytes, cudaStream_t st) {
  if (int rc = rotor_common_checks(gens, dt, S, B, T, N, D, basis)) return rc;
  if (int rc = check_heads(fn, N, H)) return rc;
  if (Mc_in && D != 16) return fail(CSN_ERR_UNSUPPORTED, fn, "the rotor cache is for D = 16");
  if (B * T * N == 0) return zero_ddt(ddt, B * T * H, st);
  if (!X || !dX || !dgens || !ddt || !dS || (gamma && !dgamma))
    return fail(CSN_ERR_INVALID, fn, "missing X, dX or a gradient output");
  if (!aligned16(X) || !aligned16(dX) || !aligned16(dS) || (h0 && !aligned16(h0)) ||
      (dh0 && !aligned16(dh0)) || (Mc_in && !aligned16(Mc_in)))
    return fail(CSN_ERR_INVALID, fn, "pointers must be 16-byte aligned");
  if (dh0 && !h0) return fail(CSN_ERR_INVALID, fn, "dh0 needs h0");
  Plan p = make_plan(B, T, N, D, true);
  Workspace ws;
  if (reuse) {
    const size_t need = plan_bytes(p);
    if (need > 256 && (!workspace || workspace_bytes < need))
      return fail(CSN_ERR_INVALID, fn, "needs the forward's workspace (csn_rotor_scan_workspace_bytes)");
    ws.base = static_cast<float*>(workspace);
  } else if (int rc = get_ws(ws, workspace, workspace_bytes, plan_bytes(p), st)) {
    return rc;
  }
  ScanArgs a{};
  a.gens = gens; a.dt = dt; a.gamma = gamma; a.S = S; a.h0 = h0; a.X = X; a.dX = dX;
  a.dgens = dgens; a.ddt = ddt; a.dgamma = dgamma; a.dC = dS; a.dh0 = dh0;
  a.B = B; a.T = T; a.N = N;
  a.dtH = H;
  a.Mc_in = Mc_in;
  a.reuse_P = reuse ? 1 : 0;
  bind_ws(a, p, ws.base, D);
  if (D == 16) return scan16_dispatch(a, SRC_ROTOR, basis, gamma != nullptr, two_sided != 0, true, st);
  return dispatch(a, D, SRC_ROTOR, basis, gamma != nullptr, two_sided != 0, true, st);
}

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

}  // namespace

extern "C" int csn_rotor_scan_fwd(const float* gens, const float* dt, const float* gamma,
                                  const float* S, const float* h0, float* X, int64_t B, int64_t T,
                                  int64_t N, int D, int basis, int two_sided, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  return rotor_fwd_impl("csn_rotor_scan_fwd", gens, dt, gamma, S, h0, X, nullptr, B, T, N, 1, D, basis,
                        two_sided, workspace, workspace_bytes, as_stream(stream));
}

extern "C" int csn_rotor_scan_bwd(const float* gens, const float* dt, const float* gamma,
                                  const float* S, const float* h0, const float* X,
                                  const float* dX, float* dgens, float* ddt, float* dgamma,
                                  float* dS, float* dh0, int64_t B, int64_t T, int64_t N, int D,
                                  int basis, int two_sided, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  return rotor_bwd_impl("csn_rotor_scan_bwd", gens, dt, gamma, S, h0, X, dX, nullptr, dgens, ddt, dgamma,
                        dS, dh0, B, T, N, 1, D, basis, two_sided, false, workspace, workspace_bytes,
                        as_stream(stream));
}

// ======================================================= backward after a forward
// csn_rotor_scan_bwd on the workspace its forward used: the chunk products P_j that the
// forward's reduce pass left in it are the ones the backward carry needs, so the backward
// reduce pass computes only the gradient aggregates.
extern "C" int csn_rotor_scan_bwd_reuse(const float* gens, const float* dt, const float* gamma,
                                        const float* S, const float* h0, const float* X,
                                        const float* dX, float* dgens, float* ddt, float* dgamma,
                                        float* dS, float* dh0, int64_t B, int64_t T, int64_t N,
                                        int D, int basis, int two_sided, void* workspace,
                                        size_t workspace_bytes, void* stream) {
  return rotor_bwd_impl("csn_rotor_scan_bwd_reuse", gens, dt, gamma, S, h0, X, dX, nullptr, dgens, ddt,
                        dgamma, dS, dh0, B, T, N, 1, D, basis, two_sided, true, workspace,
                        workspace_bytes, as_stream(stream));
}

// ======================================================= rotor cache (D = 16)
// The forward stores every step's M_t = sqrt(a_t) Q_t in Mcache ([B, T, N, 16, 16], the
// layout of S); the backward given the same Mcache loads the rotors instead of rebuilding
// them, and so does the forward's apply pass.  Three of the four passes then skip the
// Cayley transform, for 1 KB of extra HBM traffic per element per pass.
extern "C" int csn_rotor_scan_fwd_cached(const float* gens, const float* dt, const float* gamma,
                                         const float* S, const float* h0, float* X, float* Mcache,
                                         int64_t B, int64_t T, int64_t N, int D, int basis,
                                         int two_sided, void* workspace, size_t workspace_bytes,
                                         void* stream) {
  if (D != 16) {
    if (int rc = rotor_common_checks(gens, dt, S, B, T, N, D, basis)) return rc;
    return set_error(CSN_ERR_UNSUPPORTED, "csn_rotor_scan_fwd_cached: the rotor cache is for D = 16");
  }
  if (B * T * N > 0 && !Mcache)
    return set_error(CSN_ERR_INVALID, "csn_rotor_scan_fwd_cached: Mcache is required");
  return rotor_fwd_impl("csn_rotor_scan_fwd_cached", gens, dt, gamma, S, h0, X, Mcache, B, T, N, 1, D,
                        basis, two_sided, workspace, workspace_bytes, as_stream(stream));
}

extern "C" int csn_rotor_scan_bwd_cached(const float* gens, const float* dt, const float* gamma,
                                         const float* S, const float* h0, const float* X,
                                         const float* dX, const float* Mcache, float* dgens,
                                         float* ddt, float* dgamma, float* dS, float* dh0, int64_t B,
                                         int64_t T, int64_t N, int D, int basis, int two_sided,
                                         void* workspace, size_t workspace_bytes, void* stream) {
  if (D != 16) {
    if (int rc = rotor_common_checks(gens, dt, S, B, T, N, D, basis)) return rc;
    return set_error(CSN_ERR_UNSUPPORTED, "csn_rotor_scan_bwd_cached: the rotor cache is for D = 16");
  }
  if (B * T * N > 0 && !Mcache)
    return set_error(CSN_ERR_INVALID, "csn_rotor_scan_bwd_cached: Mcache is required");
  return rotor_bwd_impl("csn_rotor_scan_bwd_cached", gens, dt, gamma, S, h0, X, dX, Mcache, dgens, ddt,
                        dgamma, dS, dh0, B, T, N, 1, D, basis, two_sided, false, workspace,
                        workspace_bytes, as_stream(stream));
}

// ======================================================= multi-head layout (per-head dt)
// The H * Nh channels are H heads of Nh neurons with one dt per (b, t, head): the same
// recurrence as folding the heads into the batch ([B * H, T, Nh]) and broadcasting each
// head's dt over its neurons, read in place from the [B, T, H, Nh, ...] layout.
extern "C" int csn_rotor_scan_heads_fwd(const float* gens, const float* dt, const float* gamma,
                                        const float* S, const float* h0, float* X, float* Mcache,
                                        int64_t B, int64_t T, int64_t H, int64_t Nh, int D, int basis,
                                        int two_sided, void* workspace, size_t workspace_bytes,
                                        void* stream) {
  if (H < 0 || Nh < 0) return set_error(CSN_ERR_INVALID, "csn_rotor_scan_heads_fwd: negative dimension");
  return rotor_fwd_impl("csn_rotor_scan_heads_fwd", gens, dt, gamma, S, h0, X, Mcache, B, T, H * Nh, H, D,
                        basis, two_sided, workspace, workspace_bytes, as_stream(stream));
}

extern "C" int csn_rotor_scan_heads_bwd(const float* gens, const float* dt, const float* gamma,
                                        const float* S, const float* h0, const float* X,
                                        const float* dX, const float* Mcache, float* dgens,
                                        float* ddt, float* dgamma, float* dS, float* dh0, int64_t B,
                                        int64_t T, int64_t H, int64_t Nh, int D, int basis,
                                        int two_sided, int reuse, void* workspace,
                                        size_t workspace_bytes, void* stream) {
  if (H < 0 || Nh < 0) return set_error(CSN_ERR_INVALID, "csn_rotor_scan_heads_bwd: negative dimension");
  return rotor_bwd_impl("csn_rotor_scan_heads_bwd", gens, dt, gamma, S, h0, X, dX, Mcache, dgens, ddt,
                        dgamma, dS, dh0, B, T, H * Nh, H, D, basis, two_sided, reuse != 0,
                        workspace, workspace_bytes, as_stream(stream));
}

// ======================================================= no-allocation forward variant
//
// csn_rotor_scan_fwd_noalloc is csn_rotor_scan_fwd for callers that must not allocate
// device memory: hosts that reserve the whole GPU through their own pool (so a library
// cudaMalloc either fails or eats their budget) and serving loops where allocating
// after start-up is forbidden.  The scratch that the chunked scan needs (chunk
// aggregates and carries) lives in the file-scope array below instead of a
// caller-provided or cudaMallocAsync'd workspace.  Every GPU that loads this library
// holds the array until the process exits.
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;  // 32 MiB per device
constexpr int kNoAllocMaxDevices = 64;

}  // namespace

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device.  In host code the
// symbol name is only a host-side stand-in, so the address is looked up once per
// device (with that device current) and cached.
int noalloc_scratch(float** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_cuda_error(e, "csn_rotor_scan_fwd_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return set_error(CSN_ERR_UNSUPPORTED, "csn_rotor_scan_fwd_noalloc: device ordinal above 63");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess)
      return set_cuda_error(e, "csn_rotor_scan_fwd_noalloc: cudaGetSymbolAddress(scratch)");
    g_noalloc_ptr[dev] = p;
  }
  *out = static_cast<float*>(g_noalloc_ptr[dev]);
  return CSN_OK;
}

}  // namespace

extern "C" int csn_rotor_scan_fwd_noalloc(const float* gens, const float* dt, const float* gamma,
                                          const float* S, const float* h0, float* X, int64_t B,
                                          int64_t T, int64_t N, int D, int basis, int two_sided,
                                          void* stream) {
  if (int rc = rotor_common_checks(gens, dt, S, B, T, N, D, basis)) return rc;
  if (B * T * N == 0) return CSN_OK;
  if (!X || !aligned16(X) || (h0 && !aligned16(h0)))
    return set_error(CSN_ERR_INVALID, "csn_rotor_scan_fwd_noalloc: X missing or misaligned");
  // Same chunking as csn_rotor_scan_fwd, so both entry points give identical results.
  Plan p = make_plan(B, T, N, D, false);
  if (plan_bytes(p) > kNoAllocScratchBytes)
    return set_error(CSN_ERR_INVALID,
                     "csn_rotor_scan_fwd_noalloc: problem needs more than the 32 MiB static scratch "
                     "(csn_scan_workspace_bytes(B, T, N, D) must be <= 33554432); use "
                     "csn_rotor_scan_fwd with a workspace instead");
  float* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  ScanArgs a{};
  a.gens = gens; a.dt = dt; a.gamma = gamma; a.S = S; a.h0 = h0; a.out = X;
  a.B = B; a.T = T; a.N = N;
  bind_ws(a, p, scratch, D);
  if (D == 16) return scan16_dispatch(a, SRC_ROTOR, basis, gamma != nullptr, two_sided != 0, false, st);
  return dispatch(a, D, SRC_ROTOR, basis, gamma != nullptr, two_sided != 0, false, st);
}

// ================================================================ O(1) state step
// One recurrence step applied in place to a carried state: h <- M h M^T + C
// (one-sided: M h + C), with (M, C) built from this step's generators, dt, gamma and S.
// This is the T = 1 case of the fused scan with h0 = h; a single-chunk plan needs no
// scratch, so the call allocates nothing and launches one kernel.
static int rotor_step_impl(const float* gens, const float* dt, const float* gamma, const float* S,
                           float* h, int64_t B, int64_t N, int D, int basis, int two_sided,
                           bool chained, void* stream) {
  if (int rc = rotor_common_checks(gens, dt, S, B, 1, N, D, basis)) return rc;
  if (B * N == 0) return CSN_OK;
  if (!h || !aligned16(h)) return set_error(CSN_ERR_INVALID, "csn_rotor_step: h missing or misaligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (D == 8 && basis == BASIS_TRIU)
    return scan8_rotor_step(gens, dt, gamma, S, h, B, N, two_sided != 0, chained, st);
  Plan p = make_plan(B, 1, N, D, false);
  ScanArgs a{};
  a.gens = gens; a.dt = dt; a.gamma = gamma; a.S = S; a.h0 = h; a.out = h;
  a.B = B; a.T = 1; a.N = N;
  bind_ws(a, p, nullptr, D);
  if (D == 16) return scan16_dispatch(a, SRC_ROTOR, basis, gamma != nullptr, two_sided != 0, false, st);
  return dispatch(a, D, SRC_ROTOR, basis, gamma != nullptr, two_sided != 0, false, st);
}

extern "C" int csn_rotor_step(const float* gens, const float* dt, const float* gamma,
                              const float* S, float* h, int64_t B, int64_t N, int D, int basis,
                              int two_sided, void* stream) {
  return rotor_step_impl(gens, dt, gamma, S, h, B, N, D, basis, two_sided, false, stream);
}

// The same step for a chain of steps on one stream whose inputs are all in place before the
// chain starts (a captured decode loop): D = 8 with the triu basis launches with programmatic
// stream serialization, so each step builds its rotor while the previous step finishes and
// reads the state only once that step has completed.  Other D and bases launch as
// csn_rotor_step does.
extern "C" int csn_rotor_step_chained(const float* gens, const float* dt, const float* gamma,
                                      const float* S, float* h, int64_t B, int64_t N, int D,
                                      int basis, int two_sided, void* stream) {
  return rotor_step_impl(gens, dt, gamma, S, h, B, N, D, basis, two_sided, true, stream);
}

// ======================================================= sequence-parallel shard aggregates
// A time shard [t0, t1) of every sequence, summarised for the cross-shard carry exchange:
//   forward:  P = M_{t1-1} ... M_{t0},  c = final state of the shard scanned from zero
//   backward: c' = gradient that leaves the shard at its first step when no gradient
//             enters from the right (the shard's dh0 with zero right carry)
// A shard's carry-in is then the scan of the earlier shards' (P, c) pairs, and its
// gradient carry-in the reverse scan of the later shards' (P^T, c') pairs.
// The aggregate calls keep every chunk's aggregate in the workspace, so that the
// *_resume calls on the same inputs run only the carry and apply passes afterwards.
// The workspace also holds the per-(b, t, n) ddt partials of the backward resume.
static Plan agg_plan(int64_t B, int64_t T, int64_t N, int D) {
  Plan p = make_plan(B, T, N, D, true);
  if (p.nchunks < 1) p.nchunks = 1;
  p.agg_floats = (size_t)3 * B * N * p.nchunks * D * D;
  return p;
}

static size_t agg_bytes(int64_t B, int64_t T, int64_t N, int D) { return plan_bytes(agg_plan(B, T, N, D)); }

extern "C" size_t csn_rotor_scan_aggregate_workspace_bytes(int64_t B, int64_t T, int64_t N, int D) {
  if (B < 0 || T < 0 || N < 0 || D < 1) return 0;
  return agg_bytes(B, T, N, D);
}

static int run_aggregate(bool bwd, const float* gens, const float* dt, const float* gamma,
                         const float* S, const float* dX, float* P_out, float* c_out, int64_t B,
                         int64_t T, int64_t N, int D, int basis, int two_sided, void* workspace,
                         size_t workspace_bytes, void* stream) {
  if (int rc = rotor_common_checks(gens, dt, bwd ? dX : S, B, T, N, D, basis)) return rc;
  if (B * N == 0) return CSN_OK;
  if (T == 0) return set_error(CSN_ERR_INVALID, "shard aggregate: empty shard (T = 0)");
  if (!c_out || !aligned16(c_out) || (P_out && !aligned16(P_out)))
    return set_error(CSN_ERR_INVALID, "shard aggregate: outputs missing or misaligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Plan p = agg_plan(B, T, N, D);
  Workspace ws;
  if (int rc = get_ws(ws, workspace, workspace_bytes, plan_bytes(p), st)) return rc;
  ScanArgs a{};
  a.gens = gens; a.dt = dt; a.gamma = gamma; a.S = S; a.dX = dX;
  a.B = B; a.T = T; a.N = N;
  a.agg_mode = 1; a.P_out = P_out; a.c_out = c_out;
  bind_ws(a, p, ws.base, D);
  if (D == 16) return scan16_dispatch(a, SRC_ROTOR, basis, gamma != nullptr, two_sided != 0, bwd, st);
  return dispatch(a, D, SRC_ROTOR, basis, gamma != nullptr, two_sided != 0, bwd, st);
}

extern "C" int csn_rotor_scan_aggregate(const float* gens, const float* dt, const float* gamma,
                                        const float* S, float* P_out, float* c_out, int64_t B,
                                        int64_t T, int64_t N, int D, int basis, int two_sided,
                                        void* workspace, size_t workspace_bytes, void* stream) {
  if (!P_out) return set_error(CSN_ERR_INVALID, "csn_rotor_scan_aggregate: P_out is required");
  return run_aggregate(false, gens, dt, gamma, S, nullptr, P_out, c_out, B, T, N, D, basis,
                       two_sided, workspace, workspace_bytes, stream);
}

extern "C" int csn_rotor_scan_bwd_aggregate(const float* gens, const float* dt, const float* gamma,
                                            const float* dX, float* c_out, int64_t B, int64_t T,
                                            int64_t N, int D, int basis, int two_sided,
                                            void* workspace, size_t workspace_bytes, void* stream) {
  return run_aggregate(true, gens, dt, gamma, nullptr, dX, nullptr, c_out, B, T, N, D, basis,
                       two_sided, workspace, workspace_bytes, stream);
}

// Resume: the shard's carry and apply passes from the chunk aggregates that the
// matching aggregate call left in `workspace` (same inputs, same shape, same stream
// order).  The workspace is required: it is where those aggregates live.
static int resume_ws(void* workspace, size_t workspace_bytes, int64_t B, int64_t T, int64_t N, int D) {
  if (!workspace || workspace_bytes < agg_bytes(B, T, N, D))
    return set_error(CSN_ERR_INVALID,
                     "resume: needs the workspace of the matching aggregate call "
                     "(csn_rotor_scan_aggregate_workspace_bytes)");
  return CSN_OK;
}

extern "C" int csn_rotor_scan_fwd_resume(const float* gens, const float* dt, const float* gamma,
                                         const float* S, const float* h0, float* X, int64_t B,
                                         int64_t T, int64_t N, int D, int basis, int two_sided,
                                         void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = rotor_common_checks(gens, dt, S, B, T, N, D, basis)) return rc;
  if (B * T * N == 0) return CSN_OK;
  if (!X || !aligned16(X) || (h0 && !aligned16(h0)))
    return set_error(CSN_ERR_INVALID, "csn_rotor_scan_fwd_resume: X missing or misaligned");
  if (int rc = resume_ws(workspace, workspace_bytes, B, T, N, D)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Plan p = agg_plan(B, T, N, D);
  ScanArgs a{};
  a.gens = gens; a.dt = dt; a.gamma = gamma; a.S = S; a.h0 = h0; a.out = X;
  a.B = B; a.T = T; a.N = N;
  a.agg_mode = 2;
  bind_ws(a, p, static_cast<float*>(workspace), D);
  if (D == 16) return scan16_dispatch(a, SRC_ROTOR, basis, gamma != nullptr, two_sided != 0, false, st);
  return dispatch(a, D, SRC_ROTOR, basis, gamma != nullptr, two_sided != 0, false, st);
}

extern "C" int csn_rotor_scan_bwd_resume(const float* gens, const float* dt, const float* gamma,
                                         const float* S, const float* h0, const float* X,
                                         const float* dX, const float* dh_right, float* dgens,
                                         float* ddt, float* dgamma, float* dS, float* dh0,
                                         int64_t B, int64_t T, int64_t N, int D, int basis,
                                         int two_sided, void* workspace, size_t workspace_bytes,
                                         void* stream) {
  if (int rc = rotor_common_checks(gens, dt, S, B, T, N, D, basis)) return rc;
  if (B * T * N == 0) {
    if (B * T > 0 && ddt) {
      cudaError_t e = cudaMemsetAsync(ddt, 0, sizeof(float) * B * T, static_cast<cudaStream_t>(stream));
      if (e != cudaSuccess) return set_cuda_error(e, "cudaMemsetAsync(ddt)");
    }
    return CSN_OK;
  }
  if (!X || !dX || !dgens || !ddt || !dS || (gamma && !dgamma))
    return set_error(CSN_ERR_INVALID, "csn_rotor_scan_bwd_resume: missing X, dX or a gradient output");
  if (!aligned16(X) || !aligned16(dX) || !aligned16(dS) || (h0 && !aligned16(h0)) ||
      (dh0 && !aligned16(dh0)) || (dh_right && !aligned16(dh_right)))
    return set_error(CSN_ERR_INVALID, "csn_rotor_scan_bwd_resume: pointers must be 16-byte aligned");
  if (dh0 && !h0) return set_error(CSN_ERR_INVALID, "csn_rotor_scan_bwd_resume: dh0 needs h0");
  if (int rc = resume_ws(workspace, workspace_bytes, B, T, N, D)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Plan p = agg_plan(B, T, N, D);
  ScanArgs a{};
  a.gens = gens; a.dt = dt; a.gamma = gamma; a.S = S; a.h0 = h0; a.X = X; a.dX = dX;
  a.hT = dh_right;
  a.dgens = dgens; a.ddt = ddt; a.dgamma = dgamma; a.dC = dS; a.dh0 = dh0;
  a.B = B; a.T = T; a.N = N;
  a.agg_mode = 2;
  bind_ws(a, p, static_cast<float*>(workspace), D);
  if (D == 16) return scan16_dispatch(a, SRC_ROTOR, basis, gamma != nullptr, two_sided != 0, true, st);
  return dispatch(a, D, SRC_ROTOR, basis, gamma != nullptr, two_sided != 0, true, st);
}
