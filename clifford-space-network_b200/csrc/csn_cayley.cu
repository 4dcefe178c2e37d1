// csn_cayley.cu -- standalone exact Cayley transform and its adjoint.
//
//   Q = (I - Omega)^{-1} (I + Omega) = 2 (I - Omega)^{-1} - I
//   (python/clifford_cl6.py:57-68, python/clifford_cl8.py:29-45 with use_schulz=False)
//   dOmega = (I - Omega)^{-T} dQ (I + Q)^T = 0.5 (I + Q)^T dQ (I + Q)^T
// D = 4, 8: one thread per matrix, registers.  D = 16: one warp per matrix, the
// matrix in shared memory, each lane owning 8 of the 256 entries.
#include "csn_common.cuh"
#include "csn_internal.h"

namespace csn {

template <int D>
__global__ void __launch_bounds__(128) cayley_fwd_reg(const float* __restrict__ Om,
                                                      float* __restrict__ Q, int64_t count) {
  const int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (e >= count) return;
  Mat<D> A;
  load_mat(A, Om + e * D * D);
#pragma unroll
  for (int i = 0; i < D; ++i)
#pragma unroll
    for (int j = 0; j < D; ++j) A.a[i][j] = -A.a[i][j];  // (I - Om) - I
  gj_inverse_dev(A);  // (I - Om)^{-1} - I
  rotor_from_dev(A, 1.0f);
  store_mat(Q + e * D * D, A);
}

template <int D>
__global__ void __launch_bounds__(128) cayley_bwd_reg(const float* __restrict__ Q,
                                                      const float* __restrict__ dQ,
                                                      float* __restrict__ dOm, int64_t count) {
  const int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (e >= count) return;
  Mat<D> Bt, W;
  load_mat(Bt, Q + e * D * D);
  // Bt = (I + Q)^T
#pragma unroll
  for (int i = 0; i < D; ++i)
#pragma unroll
    for (int j = i; j < D; ++j) {
      const float u = Bt.a[i][j], v = Bt.a[j][i];
      Bt.a[i][j] = v + ((i == j) ? 1.0f : 0.0f);
      Bt.a[j][i] = u + ((i == j) ? 1.0f : 0.0f);
    }
  load_mat(W, dQ + e * D * D);
  lmul(Bt, W);
  rmul(W, Bt);
#pragma unroll
  for (int i = 0; i < D; ++i)
#pragma unroll
    for (int j = 0; j < D; ++j) W.a[i][j] *= 0.5f;
  store_mat(dOm + e * D * D, W);
}

// D = 16: warp per matrix.
__global__ void __launch_bounds__(128) cayley_fwd_16(const float* __restrict__ Om,
                                                     float* __restrict__ Q, int64_t count) {
  __shared__ float sh[4][256];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t e = blockIdx.x * 4 + w;
  if (e >= count) return;
  float* A = sh[w];
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const int idx = lane + 32 * q;
    A[idx] = -Om[e * 256 + idx];  // deviation form: (I - Om) - I (see gj_inverse_dev)
  }
  __syncwarp();
  for (int k = 0; k < 16; ++k) {
    const float ekk = A[k * 16 + k];
    const float inv = 1.0f / (1.0f + ekk);
    float nv[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int idx = lane + 32 * q, i = idx / 16, j = idx % 16;
      const float aij = A[idx];
      if (i == k && j == k) nv[q] = -ekk * inv;
      else if (i == k) nv[q] = aij * inv;
      else if (j == k) nv[q] = -aij * inv;
      else nv[q] = aij - A[i * 16 + k] * A[k * 16 + j] * inv;
    }
    __syncwarp();
#pragma unroll
    for (int q = 0; q < 8; ++q) A[lane + 32 * q] = nv[q];
    __syncwarp();
  }
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const int idx = lane + 32 * q;
    Q[e * 256 + idx] = fmaf(2.0f, A[idx], (idx / 16 == idx % 16) ? 1.0f : 0.0f);
  }
}

__global__ void __launch_bounds__(128) cayley_bwd_16(const float* __restrict__ Q,
                                                     const float* __restrict__ dQ,
                                                     float* __restrict__ dOm, int64_t count) {
  __shared__ float sB[4][256];
  __shared__ float sW[4][256];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t e = blockIdx.x * 4 + w;
  if (e >= count) return;
  float* Bt = sB[w];
  float* W = sW[w];
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const int idx = lane + 32 * q, i = idx / 16, j = idx % 16;
    Bt[j * 16 + i] = Q[e * 256 + idx] + ((i == j) ? 1.0f : 0.0f);  // (I + Q)^T
    W[idx] = dQ[e * 256 + idx];
  }
  __syncwarp();
  float v[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) {  // V = Bt dQ
    const int idx = lane + 32 * q, i = idx / 16, j = idx % 16;
    float acc = 0.0f;
#pragma unroll
    for (int k = 0; k < 16; ++k) acc = fmaf(Bt[i * 16 + k], W[k * 16 + j], acc);
    v[q] = acc;
  }
  __syncwarp();
#pragma unroll
  for (int q = 0; q < 8; ++q) W[lane + 32 * q] = v[q];
  __syncwarp();
#pragma unroll
  for (int q = 0; q < 8; ++q) {  // 0.5 V Bt
    const int idx = lane + 32 * q, i = idx / 16, j = idx % 16;
    float acc = 0.0f;
#pragma unroll
    for (int k = 0; k < 16; ++k) acc = fmaf(W[i * 16 + k], Bt[k * 16 + j], acc);
    dOm[e * 256 + idx] = 0.5f * acc;
  }
}

}  // namespace csn

using namespace csn;

static bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

extern "C" int csn_cayley_fwd(const float* Omega, float* Q, int64_t count, int D, void* stream) {
  if (count < 0) return set_error(CSN_ERR_INVALID, "csn_cayley_fwd: negative count");
  if (count == 0) return CSN_OK;
  if (!Omega || !Q || !a16(Omega) || !a16(Q))
    return set_error(CSN_ERR_INVALID, "csn_cayley_fwd: pointers missing or not 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (D != 4 && D != 8 && D != 16) return set_error(CSN_ERR_UNSUPPORTED, "csn_cayley_fwd: D must be 4, 8 or 16");
  const unsigned g1 = (unsigned)((count + 127) / 128), g4 = (unsigned)((count + 3) / 4);
  KernelTimer kt("cayley_fwd", st);
  switch (D) {
    case 4: cayley_fwd_reg<4><<<g1, 128, 0, st>>>(Omega, Q, count); break;
    case 8: cayley_fwd_reg<8><<<g1, 128, 0, st>>>(Omega, Q, count); break;
    case 16: cayley_fwd_16<<<g4, 128, 0, st>>>(Omega, Q, count); break;
    default: return set_error(CSN_ERR_UNSUPPORTED, "csn_cayley_fwd: D must be 4, 8 or 16");
  }
  return check_launch("csn_cayley_fwd");
}

extern "C" int csn_cayley_bwd(const float* Q, const float* dQ, float* dOmega, int64_t count, int D,
                              void* stream) {
  if (count < 0) return set_error(CSN_ERR_INVALID, "csn_cayley_bwd: negative count");
  if (count == 0) return CSN_OK;
  if (!Q || !dQ || !dOmega || !a16(Q) || !a16(dQ) || !a16(dOmega))
    return set_error(CSN_ERR_INVALID, "csn_cayley_bwd: pointers missing or not 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (D != 4 && D != 8 && D != 16) return set_error(CSN_ERR_UNSUPPORTED, "csn_cayley_bwd: D must be 4, 8 or 16");
  const unsigned g1 = (unsigned)((count + 127) / 128), g4 = (unsigned)((count + 3) / 4);
  KernelTimer kt("cayley_bwd", st);
  switch (D) {
    case 4: cayley_bwd_reg<4><<<g1, 128, 0, st>>>(Q, dQ, dOmega, count); break;
    case 8: cayley_bwd_reg<8><<<g1, 128, 0, st>>>(Q, dQ, dOmega, count); break;
    case 16: cayley_bwd_16<<<g4, 128, 0, st>>>(Q, dQ, dOmega, count); break;
    default: return set_error(CSN_ERR_UNSUPPORTED, "csn_cayley_bwd: D must be 4, 8 or 16");
  }
  return check_launch("csn_cayley_bwd");
}
