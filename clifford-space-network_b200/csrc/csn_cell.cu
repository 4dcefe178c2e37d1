// csn_cell.cu -- one recurrent step of the Clifford-LTC cell (CliffordTENNCell) and its
// exact adjoint, in the 4 x 4 matrix form of python/clifford_layer.py:50-115:
//   S_i   = sum_j W_rec[i,j] X_j + sum_k W_in[i,k] x_k
//   gamma = softplus(gamma_bias_i + 0.25 tr S_i)
//   Om    = 0.5 (S_i - S_i^T) * 0.5 dt
//   Q     = (I + Om)(I - Om) / (1 + 0.125 |Om|_F^2)
//   next  = sigmoid(-gamma dt) Q X_i Q^T + (1 - sigmoid(-gamma dt)) S_i
// prev/next [Bt, N, 16], x [Bt, in_dim], W_rec [N, N, 16], W_in [N, in_dim, 16].
// One thread per (batch row, neuron) for the pointwise part; the contractions over
// neurons and batch rows of the backward pass run as separate deterministic kernels.
#include "csn_common.cuh"
#include "csn_internal.h"

namespace csn {
namespace cell {

struct Fwd {
  Mat<4> S, Q, Om, rot;
  float dec, garg, den;
};

__device__ __forceinline__ float softplus_f(float v) { return v > 20.0f ? v : log1pf(expf(v)); }
__device__ __forceinline__ float sigmoid_f(float v) { return 1.0f / (1.0f + expf(-v)); }

__device__ __forceinline__ void forward_one(const float* __restrict__ prev, const float* __restrict__ x,
                                            const float* __restrict__ W_rec,
                                            const float* __restrict__ W_in,
                                            const float* __restrict__ gamma_bias, float dt,
                                            int64_t b, int64_t i, int64_t N, int64_t in_dim,
                                            Fwd& f, Mat<4>& Xi) {
  mat_zero(f.S);
  for (int64_t j = 0; j < N; ++j) {
    Mat<4> W, Xj;
    load_mat(W, W_rec + (i * N + j) * 16);
    load_mat(Xj, prev + (b * N + j) * 16);
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float s = f.S.a[r][c];
#pragma unroll
        for (int k = 0; k < 4; ++k) s = fmaf(W.a[r][k], Xj.a[k][c], s);
        f.S.a[r][c] = s;
      }
  }
  for (int64_t k = 0; k < in_dim; ++k) add_scaled_mat(f.S, W_in + (i * in_dim + k) * 16, __ldg(x + b * in_dim + k));
  const float tr = f.S.a[0][0] + f.S.a[1][1] + f.S.a[2][2] + f.S.a[3][3];
  f.garg = __ldg(gamma_bias + i) + 0.25f * tr;
  const float gam = softplus_f(f.garg);
  float nrm = 0.0f;
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      f.Om.a[r][c] = 0.5f * (f.S.a[r][c] - f.S.a[c][r]) * (0.5f * dt);
      nrm = fmaf(f.Om.a[r][c], f.Om.a[r][c], nrm);
    }
  f.den = 1.0f + 0.25f * (0.5f * nrm);
  Mat<4> Pm, Mn;
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float id = (r == c) ? 1.0f : 0.0f;
      Pm.a[r][c] = id + f.Om.a[r][c];
      Mn.a[r][c] = id - f.Om.a[r][c];
    }
  f.Q = Pm;
  rmul(f.Q, Mn);
  const float inv = 1.0f / f.den;
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) f.Q.a[r][c] *= inv;
  load_mat(Xi, prev + (b * N + i) * 16);
  f.rot = Xi;
  lmul(f.Q, f.rot);
  rmulT(f.rot, f.Q);
  f.dec = sigmoid_f(-gam * dt);
}

__global__ void __launch_bounds__(128) cell_fwd_kernel(const float* __restrict__ prev,
                                                       const float* __restrict__ x,
                                                       const float* __restrict__ W_rec,
                                                       const float* __restrict__ W_in,
                                                       const float* __restrict__ gamma_bias,
                                                       float dt, float* __restrict__ next,
                                                       int64_t Bt, int64_t N, int64_t in_dim) {
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (tid >= Bt * N) return;
  const int64_t b = tid / N, i = tid % N;
  Fwd f;
  Mat<4> Xi;
  forward_one(prev, x, W_rec, W_in, gamma_bias, dt, b, i, N, in_dim, f, Xi);
  Mat<4> out;
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) out.a[r][c] = f.dec * f.rot.a[r][c] + (1.0f - f.dec) * f.S.a[r][c];
  store_mat(next + tid * 16, out);
}

// Pointwise adjoint: writes dS [Bt,N,16], the self part of dprev, and d(gamma arg).
__global__ void __launch_bounds__(128) cell_bwd_point_kernel(
    const float* __restrict__ prev, const float* __restrict__ x, const float* __restrict__ W_rec,
    const float* __restrict__ W_in, const float* __restrict__ gamma_bias, float dt,
    const float* __restrict__ dnext, float* __restrict__ dS_out, float* __restrict__ dself,
    float* __restrict__ darg_out, int64_t Bt, int64_t N, int64_t in_dim) {
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (tid >= Bt * N) return;
  const int64_t b = tid / N, i = tid % N;
  Fwd f;
  Mat<4> Xi, G;
  forward_one(prev, x, W_rec, W_in, gamma_bias, dt, b, i, N, in_dim, f, Xi);
  load_mat(G, dnext + tid * 16);
  // next = dec rot + (1 - dec) S
  float ddec = 0.0f;
  Mat<4> dS, dR;
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      ddec = fmaf(G.a[r][c], f.rot.a[r][c] - f.S.a[r][c], ddec);
      dS.a[r][c] = (1.0f - f.dec) * G.a[r][c];
      dR.a[r][c] = f.dec * G.a[r][c];
    }
  // dec = sigmoid(-gamma dt), gamma = softplus(arg)
  const float dgam = ddec * f.dec * (1.0f - f.dec) * (-dt);
  const float darg = dgam * sigmoid_f(f.garg);
  darg_out[tid] = darg;
#pragma unroll
  for (int d = 0; d < 4; ++d) dS.a[d][d] += 0.25f * darg;
  // rot = Q X Q^T:  dQ = dR Q X^T + dR^T Q X;  dX_self = Q^T dR Q
  Mat<4> dQ, t1, t2;
  t1 = dR; rmul(t1, f.Q); rmulT(t1, Xi);      // dR Q X^T
  t2 = Xi; lmul(f.Q, t2);                      // Q X
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float s = t1.a[r][c];
#pragma unroll
      for (int k = 0; k < 4; ++k) s = fmaf(dR.a[k][r], t2.a[k][c], s);  // dR^T (Q X)
      dQ.a[r][c] = s;
    }
  Mat<4> ds = dR;
  lmulT(f.Q, ds);
  rmul(ds, f.Q);
  store_mat(dself + tid * 16, ds);
  // Q = P Mn / den, P = I + Om, Mn = I - Om, den = 1 + 0.125 |Om|^2
  const float inv = 1.0f / f.den;
  float dden = 0.0f;
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) dden = fmaf(dQ.a[r][c], f.Q.a[r][c], dden);
  dden = -dden * inv;
  Mat<4> Pm, Mn, dP, dMn;
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float id = (r == c) ? 1.0f : 0.0f;
      Pm.a[r][c] = id + f.Om.a[r][c];
      Mn.a[r][c] = id - f.Om.a[r][c];
      dQ.a[r][c] *= inv;
    }
  dP = dQ; rmulT(dP, Mn);     // (dQ/den) Mn^T
  dMn = dQ; lmulT(Pm, dMn);   // P^T (dQ/den)
  // dOm = dP - dMn + dden * 0.25 Om ; Om = 0.25 dt (S - S^T)
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) t1.a[r][c] = dP.a[r][c] - dMn.a[r][c] + dden * 0.25f * f.Om.a[r][c];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) dS.a[r][c] += 0.25f * dt * (t1.a[r][c] - t1.a[c][r]);
  store_mat(dS_out + tid * 16, dS);
}

// dprev[b, j] = dself[b, j] + sum_i W_rec[i, j]^T dS[b, i];  one thread per (b, j)
__global__ void __launch_bounds__(128) cell_bwd_dprev_kernel(const float* __restrict__ W_rec,
                                                             const float* __restrict__ dS,
                                                             const float* __restrict__ dself,
                                                             float* __restrict__ dprev, int64_t Bt,
                                                             int64_t N) {
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (tid >= Bt * N) return;
  const int64_t b = tid / N, j = tid % N;
  Mat<4> acc;
  load_mat(acc, dself + tid * 16);
  for (int64_t i = 0; i < N; ++i) {
    Mat<4> W, G;
    load_mat(W, W_rec + (i * N + j) * 16);
    load_mat(G, dS + (b * N + i) * 16);
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float s = acc.a[r][c];
#pragma unroll
        for (int k = 0; k < 4; ++k) s = fmaf(W.a[k][r], G.a[k][c], s);
        acc.a[r][c] = s;
      }
  }
  store_mat(dprev + tid * 16, acc);
}

// dx[b, k] = sum_i <W_in[i, k], dS[b, i]>;  one thread per (b, k)
__global__ void __launch_bounds__(128) cell_bwd_dx_kernel(const float* __restrict__ W_in,
                                                          const float* __restrict__ dS,
                                                          float* __restrict__ dx, int64_t Bt,
                                                          int64_t N, int64_t in_dim) {
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (tid >= Bt * in_dim) return;
  const int64_t b = tid / in_dim, k = tid % in_dim;
  float s = 0.0f;
  for (int64_t i = 0; i < N; ++i) {
    Mat<4> G;
    load_mat(G, dS + (b * N + i) * 16);
    s += mat_dot_global(G, W_in + (i * in_dim + k) * 16);
  }
  dx[tid] = s;
}

// Parameter gradients, reduced over the batch in a fixed order (deterministic):
//   dW_rec[i, j] = sum_b dS[b, i] X[b, j]^T   (threads 0 .. N*N-1)
//   dW_in[i, k]  = sum_b dS[b, i] x[b, k]     (next N*in_dim threads)
//   dgamma_bias[i] = sum_b darg[b, i]         (last N threads)
__global__ void __launch_bounds__(128) cell_bwd_params_kernel(
    const float* __restrict__ prev, const float* __restrict__ x, const float* __restrict__ dS,
    const float* __restrict__ darg, float* __restrict__ dW_rec, float* __restrict__ dW_in,
    float* __restrict__ dgb, int64_t Bt, int64_t N, int64_t in_dim) {
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t n1 = N * N, n2 = N * in_dim;
  if (tid < n1) {
    const int64_t i = tid / N, j = tid % N;
    Mat<4> acc;
    mat_zero(acc);
    for (int64_t b = 0; b < Bt; ++b) {
      Mat<4> G, X;
      load_mat(G, dS + (b * N + i) * 16);
      load_mat(X, prev + (b * N + j) * 16);
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float s = acc.a[r][c];
#pragma unroll
          for (int k = 0; k < 4; ++k) s = fmaf(G.a[r][k], X.a[c][k], s);
          acc.a[r][c] = s;
        }
    }
    if (dW_rec) store_mat(dW_rec + tid * 16, acc);
  } else if (tid < n1 + n2) {
    const int64_t q = tid - n1, i = q / in_dim, k = q % in_dim;
    Mat<4> acc;
    mat_zero(acc);
    for (int64_t b = 0; b < Bt; ++b) add_scaled_mat(acc, dS + (b * N + i) * 16, __ldg(x + b * in_dim + k));
    if (dW_in) store_mat(dW_in + q * 16, acc);
  } else if (tid < n1 + n2 + N) {
    const int64_t i = tid - n1 - n2;
    float s = 0.0f;
    for (int64_t b = 0; b < Bt; ++b) s += darg[b * N + i];
    if (dgb) dgb[i] = s;
  }
}

}  // namespace cell
}  // namespace csn

using namespace csn;

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

extern "C" size_t csn_cell_workspace_bytes(int64_t Bt, int64_t N) {
  if (Bt < 0 || N < 0) return 0;
  return (size_t)Bt * N * (16 + 16 + 1) * sizeof(float) + 512;
}

extern "C" int csn_cell_fwd(const float* prev, const float* x, const float* W_rec, const float* W_in,
                            const float* gamma_bias, float dt, float* next, int64_t Bt, int64_t N,
                            int64_t in_dim, void* stream) {
  if (Bt < 0 || N < 0 || in_dim < 0) return set_error(CSN_ERR_INVALID, "csn_cell_fwd: negative size");
  if (Bt * N == 0) return CSN_OK;
  if (!prev || !W_rec || !gamma_bias || !next || (in_dim > 0 && (!x || !W_in)))
    return set_error(CSN_ERR_INVALID, "csn_cell_fwd: missing pointer");
  if (!al16(prev) || !al16(W_rec) || !al16(next) || (in_dim > 0 && !al16(W_in)))
    return set_error(CSN_ERR_INVALID, "csn_cell_fwd: 16-byte alignment required");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t n = Bt * N;
  KernelTimer kt("cell_fwd", st);
  cell::cell_fwd_kernel<<<(unsigned)((n + 127) / 128), 128, 0, st>>>(prev, x, W_rec, W_in, gamma_bias,
                                                                      dt, next, Bt, N, in_dim);
  return check_launch("csn_cell_fwd");
}

extern "C" int csn_cell_bwd(const float* prev, const float* x, const float* W_rec, const float* W_in,
                            const float* gamma_bias, float dt, const float* dnext, float* dprev,
                            float* dx, float* dW_rec, float* dW_in, float* dgamma_bias, int64_t Bt,
                            int64_t N, int64_t in_dim, void* workspace, size_t workspace_bytes,
                            void* stream) {
  if (Bt < 0 || N < 0 || in_dim < 0) return set_error(CSN_ERR_INVALID, "csn_cell_bwd: negative size");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (Bt * N == 0) return CSN_OK;
  if (!prev || !W_rec || !gamma_bias || !dnext || !dprev || (in_dim > 0 && (!x || !W_in)))
    return set_error(CSN_ERR_INVALID, "csn_cell_bwd: missing pointer");
  if (!al16(prev) || !al16(W_rec) || !al16(dnext) || !al16(dprev) || (in_dim > 0 && !al16(W_in)) ||
      (dW_rec && !al16(dW_rec)) || (dW_in && !al16(dW_in)))
    return set_error(CSN_ERR_INVALID, "csn_cell_bwd: 16-byte alignment required");
  const size_t need = csn_cell_workspace_bytes(Bt, N);
  float* ws = nullptr;
  bool owned = false;
  if (workspace) {
    if (workspace_bytes < need) return set_error(CSN_ERR_INVALID, "csn_cell_bwd: workspace too small");
    ws = static_cast<float*>(workspace);
  } else {
    cudaError_t e = cudaMallocAsync(reinterpret_cast<void**>(&ws), need, st);
    if (e != cudaSuccess) return set_cuda_error(e, "csn_cell_bwd: cudaMallocAsync");
    owned = true;
  }
  float* base = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(ws) + 255) & ~uintptr_t(255));
  float* dS = base;
  float* dself = dS + Bt * N * 16;
  float* darg = dself + Bt * N * 16;
  const int64_t n = Bt * N;
  {
    KernelTimer kt("cell_bwd", st);
    cell::cell_bwd_point_kernel<<<(unsigned)((n + 127) / 128), 128, 0, st>>>(
        prev, x, W_rec, W_in, gamma_bias, dt, dnext, dS, dself, darg, Bt, N, in_dim);
    cell::cell_bwd_dprev_kernel<<<(unsigned)((n + 127) / 128), 128, 0, st>>>(W_rec, dS, dself, dprev,
                                                                             Bt, N);
    if (dx && in_dim > 0)
      cell::cell_bwd_dx_kernel<<<(unsigned)((Bt * in_dim + 127) / 128), 128, 0, st>>>(W_in, dS, dx, Bt,
                                                                                     N, in_dim);
    const int64_t np = N * N + N * in_dim + N;
    cell::cell_bwd_params_kernel<<<(unsigned)((np + 127) / 128), 128, 0, st>>>(
        prev, x, dS, darg, dW_rec, dW_in, dgamma_bias, Bt, N, in_dim);
  }
  int rc = check_launch("csn_cell_bwd");
  if (owned) cudaFreeAsync(ws, st);
  return rc;
}
