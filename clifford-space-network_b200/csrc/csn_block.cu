// csn_block.cu -- the row / per-state kernels of the Clifford blocks around the scan.
//
// Event spike on the scan output (python/clifford_scan.py:90-116 SurrogateSpikeFunction,
// applied to the Frobenius energy of each state matrix, python/clifford_cl6.py:174-176):
//   e = ||X||_F,  s = [e - thr >= 0],  Xs = s X
// and its surrogate adjoint (fast sigmoid, 1 / (1 + beta |e - thr|)^2):
//   dX = s dXs + (<dXs, X> sg / e) X          (the norm's gradient is 0 where e = 0)
// One D x D state is spread over min(32, D*D/4) lanes of a warp as float4 columns, so loads
// and stores are 16-byte and coalesced; the energy and <dXs, X> are reduced by shuffles.
//
// LayerNorm over the last dimension (nn.LayerNorm of every block, eps as given):
//   y = (x - mean) rstd g + b,  rstd = 1 / sqrt(var + eps)   (biased variance)
//   dx = rstd (g dy - mean(g dy) - xhat mean(g dy xhat)),  dg = sum_rows dy xhat,  db = sum_rows dy
// One warp per row, the row in registers (C <= 1024, C % 4 == 0); the parameter gradients
// are summed per CTA and then over CTAs by a second kernel.
#include <cstdio>

#include "csn_common.cuh"
#include "csn_internal.h"

namespace csn {
namespace {

constexpr unsigned FULLMASK = 0xffffffffu;

__device__ __forceinline__ float dot4(const float4& a, const float4& b) {
  return a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w;
}

// ------------------------------------------------------------------------ spike
template <int DD>
struct SpikeShape {
  static constexpr int V = DD / 4;                 // float4 per state
  static constexpr int L = V < 32 ? V : 32;        // lanes per state
  static constexpr int PV = V / L;                 // float4 per lane
  static constexpr int PER_WARP = 32 / L;          // states per warp
};

template <int L>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int o = L / 2; o > 0; o >>= 1) v += __shfl_xor_sync(FULLMASK, v, o);
  return v;
}

template <int DD>
__global__ void __launch_bounds__(256) spike_fwd_kernel(const float* __restrict__ X, float* __restrict__ Xs,
                                                        int64_t n, float thr) {
  using Sh = SpikeShape<DD>;
  const int lane = threadIdx.x & 31;
  const int sub = lane % Sh::L;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t w = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); w * Sh::PER_WARP < n;
       w += warps) {
    const int64_t e = w * Sh::PER_WARP + lane / Sh::L;
    const bool live = e < n;
    const float4* src = reinterpret_cast<const float4*>(X + e * DD);
    float4 v[Sh::PV];
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < Sh::PV; ++k) {
      v[k] = live ? __ldg(src + sub + Sh::L * k) : make_float4(0.f, 0.f, 0.f, 0.f);
      ss += dot4(v[k], v[k]);
    }
    ss = group_sum<Sh::L>(ss);
    const float s = (sqrtf(ss) - thr >= 0.0f) ? 1.0f : 0.0f;
    if (live) {
      float4* dst = reinterpret_cast<float4*>(Xs + e * DD);
#pragma unroll
      for (int k = 0; k < Sh::PV; ++k)
        dst[sub + Sh::L * k] = make_float4(v[k].x * s, v[k].y * s, v[k].z * s, v[k].w * s);
    }
  }
}

template <int DD>
__global__ void __launch_bounds__(256) spike_bwd_kernel(const float* __restrict__ X, const float* __restrict__ dXs,
                                                        float* __restrict__ dX, int64_t n, float thr, float beta) {
  using Sh = SpikeShape<DD>;
  const int lane = threadIdx.x & 31;
  const int sub = lane % Sh::L;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t w = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); w * Sh::PER_WARP < n;
       w += warps) {
    const int64_t e = w * Sh::PER_WARP + lane / Sh::L;
    const bool live = e < n;
    const float4* xs = reinterpret_cast<const float4*>(X + e * DD);
    const float4* gs = reinterpret_cast<const float4*>(dXs + e * DD);
    float4 v[Sh::PV], g[Sh::PV];
    float ss = 0.0f, dot = 0.0f;
#pragma unroll
    for (int k = 0; k < Sh::PV; ++k) {
      const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
      v[k] = live ? __ldg(xs + sub + Sh::L * k) : z;
      g[k] = live ? __ldg(gs + sub + Sh::L * k) : z;
      ss += dot4(v[k], v[k]);
      dot += dot4(g[k], v[k]);
    }
    ss = group_sum<Sh::L>(ss);
    dot = group_sum<Sh::L>(dot);
    const float en = sqrtf(ss);
    const float x = en - thr;
    const float s = (x >= 0.0f) ? 1.0f : 0.0f;
    const float q = 1.0f + beta * fabsf(x);
    const float de = dot * (1.0f / (q * q));    // d energy
    const float c = en > 0.0f ? de / en : 0.0f;  // norm backward: (grad / norm) X, 0 at norm 0
    if (live) {
      float4* dst = reinterpret_cast<float4*>(dX + e * DD);
#pragma unroll
      for (int k = 0; k < Sh::PV; ++k)
        dst[sub + Sh::L * k] = make_float4(g[k].x * s + c * v[k].x, g[k].y * s + c * v[k].y,
                                           g[k].z * s + c * v[k].z, g[k].w * s + c * v[k].w);
    }
  }
}

unsigned spike_grid(int64_t n, int per_warp) {
  const int64_t warps = (n + per_warp - 1) / per_warp;
  const int64_t blocks = (warps + 7) / 8;
  const int64_t cap = 148 * 16;  // grid-stride beyond 16 CTAs of 256 threads per SM
  return (unsigned)(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}

// ------------------------------------------------------------------------ LayerNorm
// NV = float4 per lane (C <= 128 * NV).
template <int NV>
__global__ void __launch_bounds__(256) ln_fwd_kernel(const float* __restrict__ x, const float* __restrict__ g,
                                                     const float* __restrict__ b, float* __restrict__ y,
                                                     float* __restrict__ mean_out, float* __restrict__ rstd_out,
                                                     int64_t R, int C, float eps) {
  const int lane = threadIdx.x & 31;
  const int C4 = C >> 2;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const float inv_c = 1.0f / (float)C;
  for (int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); r < R; r += warps) {
    const float4* xr = reinterpret_cast<const float4*>(x + r * C);
    float4 v[NV];
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int j = lane + 32 * k;
      v[k] = j < C4 ? __ldg(xr + j) : make_float4(0.f, 0.f, 0.f, 0.f);
      s += (v[k].x + v[k].y) + (v[k].z + v[k].w);
    }
    s = group_sum<32>(s);
    const float mu = s * inv_c;
    float q = 0.0f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int j = lane + 32 * k;
      if (j < C4) {
        const float a = v[k].x - mu, bb = v[k].y - mu, c = v[k].z - mu, d = v[k].w - mu;
        q += (a * a + bb * bb) + (c * c + d * d);
      }
    }
    q = group_sum<32>(q);
    const float rs = rsqrtf(q * inv_c + eps);
    float4* yr = reinterpret_cast<float4*>(y + r * C);
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int j = lane + 32 * k;
      if (j < C4) {
        const float4 gg = __ldg(reinterpret_cast<const float4*>(g) + j);
        const float4 bv = __ldg(reinterpret_cast<const float4*>(b) + j);
        yr[j] = make_float4((v[k].x - mu) * rs * gg.x + bv.x, (v[k].y - mu) * rs * gg.y + bv.y,
                            (v[k].z - mu) * rs * gg.z + bv.z, (v[k].w - mu) * rs * gg.w + bv.w);
      }
    }
    if (lane == 0) {
      mean_out[r] = mu;
      rstd_out[r] = rs;
    }
  }
}

// Row gradients and per-CTA partial sums of dg, db: part[blockIdx.x, 0:C] = dg, [C:2C] = db.
template <int NV>
__global__ void __launch_bounds__(256) ln_bwd_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                                                     const float* __restrict__ mean, const float* __restrict__ rstd,
                                                     const float* __restrict__ g, float* __restrict__ dx,
                                                     float* __restrict__ part, int64_t R, int C) {
  extern __shared__ float ln_smem[];  // [warps][2C]
  const int lane = threadIdx.x & 31;
  const int wid = threadIdx.x >> 5;
  const int C4 = C >> 2;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const float inv_c = 1.0f / (float)C;
  float4 ag[NV], ab[NV];
#pragma unroll
  for (int k = 0; k < NV; ++k) ag[k] = ab[k] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + wid; r < R; r += warps) {
    const float4* xr = reinterpret_cast<const float4*>(x + r * C);
    const float4* dr = reinterpret_cast<const float4*>(dy + r * C);
    const float mu = __ldg(mean + r), rs = __ldg(rstd + r);
    float4 xh[NV], wd[NV];
    float s1 = 0.0f, s2 = 0.0f;  // sum(g dy xhat), sum(g dy)
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int j = lane + 32 * k;
      if (j < C4) {
        const float4 xv = __ldg(xr + j), dv = __ldg(dr + j);
        const float4 gg = __ldg(reinterpret_cast<const float4*>(g) + j);
        xh[k] = make_float4((xv.x - mu) * rs, (xv.y - mu) * rs, (xv.z - mu) * rs, (xv.w - mu) * rs);
        wd[k] = make_float4(dv.x * gg.x, dv.y * gg.y, dv.z * gg.z, dv.w * gg.w);
        s1 += dot4(wd[k], xh[k]);
        s2 += (wd[k].x + wd[k].y) + (wd[k].z + wd[k].w);
        ag[k].x += dv.x * xh[k].x; ag[k].y += dv.y * xh[k].y; ag[k].z += dv.z * xh[k].z; ag[k].w += dv.w * xh[k].w;
        ab[k].x += dv.x; ab[k].y += dv.y; ab[k].z += dv.z; ab[k].w += dv.w;
      } else {
        xh[k] = wd[k] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    s1 = group_sum<32>(s1) * inv_c;
    s2 = group_sum<32>(s2) * inv_c;
    float4* o = reinterpret_cast<float4*>(dx + r * C);
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int j = lane + 32 * k;
      if (j < C4)
        o[j] = make_float4((wd[k].x - xh[k].x * s1 - s2) * rs, (wd[k].y - xh[k].y * s1 - s2) * rs,
                           (wd[k].z - xh[k].z * s1 - s2) * rs, (wd[k].w - xh[k].w * s1 - s2) * rs);
    }
  }
  // per-CTA sum of the warps' partials
  float* mine = ln_smem + wid * 2 * C;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int j = lane + 32 * k;
    if (j < C4) {
      reinterpret_cast<float4*>(mine)[j] = ag[k];
      reinterpret_cast<float4*>(mine + C)[j] = ab[k];
    }
  }
  __syncthreads();
  const int nw = blockDim.x >> 5;
  for (int c = threadIdx.x; c < 2 * C; c += blockDim.x) {
    float t = 0.0f;
    for (int w = 0; w < nw; ++w) t += ln_smem[w * 2 * C + c];
    part[(int64_t)blockIdx.x * 2 * C + c] = t;
  }
}

// dg[c] = sum_p part[p, c], db[c] = sum_p part[p, C + c]: 32 columns per CTA, its 8 warps
// sum interleaved rows and the CTA adds the 8 warp sums in a fixed order (deterministic).
__global__ void __launch_bounds__(256) ln_param_reduce_kernel(const float* __restrict__ part,
                                                              float* __restrict__ dg, float* __restrict__ db,
                                                              int P, int C) {
  __shared__ float acc[8][33];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + lane;
  float t = 0.0f;
  if (c < 2 * C)
    for (int p = wid; p < P; p += 8) t += part[(int64_t)p * 2 * C + c];
  acc[wid][lane] = t;
  __syncthreads();
  if (wid == 0 && c < 2 * C) {
    float u = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) u += acc[w][lane];
    if (c < C) {
      if (dg) dg[c] = u;
    } else if (db) {
      db[c - C] = u;
    }
  }
}

constexpr int LN_THREADS = 256;

unsigned ln_grid(int64_t R) {
  const int64_t blocks = (R + 7) / 8;
  const int64_t cap = 148 * 4;
  return (unsigned)(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int ln_check(const char* fn, int64_t R, int C) {
  if (R < 0 || C <= 0 || C % 4 != 0 || C > 1024) {
    char buf[160];
    snprintf(buf, sizeof(buf), "%s: needs R >= 0 and 0 < C <= 1024 with C %% 4 == 0", fn);
    return set_error(CSN_ERR_UNSUPPORTED, buf);
  }
  return CSN_OK;
}

}  // namespace
}  // namespace csn

using namespace csn;

extern "C" int csn_spike_fwd(const float* X, float* Xs, int64_t n, int D, float threshold, void* stream) {
  if (n < 0 || (D != 4 && D != 8 && D != 16)) return set_error(CSN_ERR_INVALID, "csn_spike_fwd: n >= 0, D in {4, 8, 16}");
  if (n == 0) return CSN_OK;
  if (!X || !Xs || !al16(X) || !al16(Xs)) return set_error(CSN_ERR_INVALID, "csn_spike_fwd: 16-byte aligned X, Xs required");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  KernelTimer kt("spike_fwd", st);
  if (D == 4) spike_fwd_kernel<16><<<spike_grid(n, SpikeShape<16>::PER_WARP), 256, 0, st>>>(X, Xs, n, threshold);
  else if (D == 8) spike_fwd_kernel<64><<<spike_grid(n, SpikeShape<64>::PER_WARP), 256, 0, st>>>(X, Xs, n, threshold);
  else spike_fwd_kernel<256><<<spike_grid(n, SpikeShape<256>::PER_WARP), 256, 0, st>>>(X, Xs, n, threshold);
  return check_launch("csn_spike_fwd");
}

extern "C" int csn_spike_bwd(const float* X, const float* dXs, float* dX, int64_t n, int D, float threshold,
                             float beta, void* stream) {
  if (n < 0 || (D != 4 && D != 8 && D != 16)) return set_error(CSN_ERR_INVALID, "csn_spike_bwd: n >= 0, D in {4, 8, 16}");
  if (n == 0) return CSN_OK;
  if (!X || !dXs || !dX || !al16(X) || !al16(dXs) || !al16(dX))
    return set_error(CSN_ERR_INVALID, "csn_spike_bwd: 16-byte aligned X, dXs, dX required");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  KernelTimer kt("spike_bwd", st);
  if (D == 4)
    spike_bwd_kernel<16><<<spike_grid(n, SpikeShape<16>::PER_WARP), 256, 0, st>>>(X, dXs, dX, n, threshold, beta);
  else if (D == 8)
    spike_bwd_kernel<64><<<spike_grid(n, SpikeShape<64>::PER_WARP), 256, 0, st>>>(X, dXs, dX, n, threshold, beta);
  else
    spike_bwd_kernel<256><<<spike_grid(n, SpikeShape<256>::PER_WARP), 256, 0, st>>>(X, dXs, dX, n, threshold, beta);
  return check_launch("csn_spike_bwd");
}

extern "C" int csn_layer_norm_fwd(const float* x, const float* weight, const float* bias, float* y, float* mean,
                                  float* rstd, int64_t R, int C, float eps, void* stream) {
  if (int rc = ln_check("csn_layer_norm_fwd", R, C)) return rc;
  if (R == 0) return CSN_OK;
  if (!x || !weight || !bias || !y || !mean || !rstd || !al16(x) || !al16(y) || !al16(weight) || !al16(bias))
    return set_error(CSN_ERR_INVALID, "csn_layer_norm_fwd: missing or misaligned pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  KernelTimer kt("layer_norm_fwd", st);
  const unsigned grid = ln_grid(R);
  if (C <= 128) ln_fwd_kernel<1><<<grid, LN_THREADS, 0, st>>>(x, weight, bias, y, mean, rstd, R, C, eps);
  else if (C <= 256) ln_fwd_kernel<2><<<grid, LN_THREADS, 0, st>>>(x, weight, bias, y, mean, rstd, R, C, eps);
  else if (C <= 512) ln_fwd_kernel<4><<<grid, LN_THREADS, 0, st>>>(x, weight, bias, y, mean, rstd, R, C, eps);
  else ln_fwd_kernel<8><<<grid, LN_THREADS, 0, st>>>(x, weight, bias, y, mean, rstd, R, C, eps);
  return check_launch("csn_layer_norm_fwd");
}

extern "C" size_t csn_layer_norm_bwd_workspace_bytes(int64_t R, int C) {
  if (R <= 0 || C <= 0) return 0;
  return (size_t)ln_grid(R) * 2 * (size_t)C * sizeof(float);
}

extern "C" int csn_layer_norm_bwd(const float* dy, const float* x, const float* mean, const float* rstd,
                                  const float* weight, float* dx, float* dweight, float* dbias, int64_t R, int C,
                                  void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = ln_check("csn_layer_norm_bwd", R, C)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (R == 0) {
    if (dweight && cudaMemsetAsync(dweight, 0, sizeof(float) * C, st) != cudaSuccess)
      return set_error(CSN_ERR_CUDA, "csn_layer_norm_bwd: cudaMemsetAsync");
    if (dbias && cudaMemsetAsync(dbias, 0, sizeof(float) * C, st) != cudaSuccess)
      return set_error(CSN_ERR_CUDA, "csn_layer_norm_bwd: cudaMemsetAsync");
    return CSN_OK;
  }
  if (!dy || !x || !mean || !rstd || !weight || !dx || !al16(dy) || !al16(x) || !al16(dx) || !al16(weight))
    return set_error(CSN_ERR_INVALID, "csn_layer_norm_bwd: missing or misaligned pointer");
  const unsigned grid = ln_grid(R);
  if (!workspace || workspace_bytes < csn_layer_norm_bwd_workspace_bytes(R, C))
    return set_error(CSN_ERR_INVALID, "csn_layer_norm_bwd: workspace smaller than csn_layer_norm_bwd_workspace_bytes");
  float* part = static_cast<float*>(workspace);
  const size_t smem = (size_t)(LN_THREADS / 32) * 2 * C * sizeof(float);  // <= 64 KB at C = 1024
  {
    KernelTimer kt("layer_norm_bwd", st);
    if (C <= 128) ln_bwd_kernel<1><<<grid, LN_THREADS, smem, st>>>(dy, x, mean, rstd, weight, dx, part, R, C);
    else if (C <= 256) ln_bwd_kernel<2><<<grid, LN_THREADS, smem, st>>>(dy, x, mean, rstd, weight, dx, part, R, C);
    else if (C <= 512) ln_bwd_kernel<4><<<grid, LN_THREADS, smem, st>>>(dy, x, mean, rstd, weight, dx, part, R, C);
    else {
      // up to 64 KB of dynamic shared memory for C in (512, 1024]
      cudaError_t e = cudaFuncSetAttribute(ln_bwd_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)((LN_THREADS / 32) * 2 * 1024 * sizeof(float)));
      if (e != cudaSuccess) return set_cuda_error(e, "csn_layer_norm_bwd: cudaFuncSetAttribute");
      ln_bwd_kernel<8><<<grid, LN_THREADS, smem, st>>>(dy, x, mean, rstd, weight, dx, part, R, C);
    }
  }
  if (dweight || dbias) {
    KernelTimer kt("layer_norm_param_reduce", st);
    ln_param_reduce_kernel<<<(unsigned)((2 * C + 31) / 32), 256, 0, st>>>(part, dweight, dbias, (int)grid, C);
  }
  return check_launch("csn_layer_norm_bwd");
}
