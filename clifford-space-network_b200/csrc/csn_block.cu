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
//
// The blocks' input chain ln_1 -> causal depthwise conv1d (kernel K, left zero padding) -> SiLU
// (python/clifford_cl6.py:140-142), fused:
//   y[b, t, c] = silu(cb[c] + sum_{j<K} cw[c, j] ln[b, t - K + 1 + j, c]),  ln rows t < 0 are 0
// One warp walks a chunk of time steps of one sequence with the last K LayerNorm rows in a
// register ring, so x is read once and neither the transposed, padded nor pre-activation
// tensors exist.  The backward walks the same chunk (plus K - 1 rows of look-ahead) with rings
// of LayerNorm rows and conv-output gradients:
//   du_t = dy_t silu'(u_t),  dln_s = sum_j cw[:, j] du_{s + K - 1 - j},  then the LayerNorm adjoint;
// conv weight / bias and LayerNorm weight / bias gradients are summed per CTA, then over CTAs.
//
// Least-action terms of the LMs (python/clifford_cl6.py:257-262) on the generator coefficients
// w[b, t, j] = 0.5 dt[b, t, head(j)] biv[b, t, j] (row of R = N * K coefficients, H heads of R / H):
//   S_kin = sum w^2,  S_smooth = sum_{t >= 1} (w_t - w_{t-1})^2
// and the adjoint for dL/de_kin, dL/de_smooth with e = c S (c given by the caller):
//   dw_t = 2 c_k g_k w_t + 2 c_s g_s ((w_t - w_{t-1}) [t >= 1] - (w_{t+1} - w_t) [t <= T - 2])
//   dbiv = 0.5 dt dw,  ddt[b, t, h] = sum_{j in head h} 0.5 biv dw
// The gradient scalars are read on the device, so no host synchronisation is needed.
//
// Projection epilogue (python/clifford_cl6.py:144-155): the generator, decay and time
// projections run as ONE GEMM whose rows hold Q = N*K + N + HT columns
// [generators | gamma | time]; the epilogue writes the scan's inputs
//   biv = raw * omega_scale[n],  gamma = softplus(raw),  dt = softplus(raw) * dt_base
// (softplus(x) = x above 20, as torch) and its adjoint writes the GEMM output's gradient in
// the same layout plus per-row partials of d omega_scale (summed by the column sum).
// Column sum: deterministic sums of the rows of a [R, C] matrix (bias gradients).
// Gate of the GGLU: y = silu(g) * u on one [R, 2F] GEMM output [g | u], and its adjoint into
// one [R, 2F] gradient (python/clifford_model.py:42-43).
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
  float t0 = 0.0f, t1 = 0.0f, t2 = 0.0f, t3 = 0.0f;  // four independent chains
  if (c < 2 * C) {
    int p = wid;
    for (; p + 24 < P; p += 32) {
      t0 += part[(int64_t)p * 2 * C + c];
      t1 += part[(int64_t)(p + 8) * 2 * C + c];
      t2 += part[(int64_t)(p + 16) * 2 * C + c];
      t3 += part[(int64_t)(p + 24) * 2 * C + c];
    }
    for (; p < P; p += 8) t0 += part[(int64_t)p * 2 * C + c];
  }
  acc[wid][lane] = (t0 + t1) + (t2 + t3);
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

// ------------------------------------------------------- ln -> causal conv -> SiLU
// C <= 128 * NV, K <= 4.
template <int NV>
__device__ __forceinline__ void load_row_params(const float* __restrict__ p, int C4, int lane, float4 (&out)[NV]) {
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int j = lane + 32 * k;
    out[k] = j < C4 ? __ldg(reinterpret_cast<const float4*>(p) + j) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// cw [C, 1, K]: tap j of the 4 channels of float4 column jc
template <int NV, int K>
__device__ __forceinline__ void load_conv_taps(const float* __restrict__ cw, int C4, int lane, float4 (&w)[K][NV]) {
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int jc = lane + 32 * k;
#pragma unroll
    for (int j = 0; j < K; ++j)
      w[j][k] = jc < C4 ? make_float4(__ldg(cw + (4 * jc + 0) * K + j), __ldg(cw + (4 * jc + 1) * K + j),
                                      __ldg(cw + (4 * jc + 2) * K + j), __ldg(cw + (4 * jc + 3) * K + j))
                        : make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

template <int NV>
__device__ __forceinline__ void load_row(const float* __restrict__ xr, int C4, int lane, float4 (&v)[NV]) {
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int j = lane + 32 * k;
    v[k] = j < C4 ? __ldg(reinterpret_cast<const float4*>(xr) + j) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// LayerNorm of one row held as v (warp-collective): out = (x - mu) rs g + b
template <int NV>
__device__ __forceinline__ void ln_vals(const float4 (&v)[NV], int C4, int lane, float inv_c, float eps,
                                        const float4 (&g)[NV], const float4 (&b)[NV], float4 (&out)[NV],
                                        float& mu, float& rs) {
  float s = 0.0f;
#pragma unroll
  for (int k = 0; k < NV; ++k) s += (v[k].x + v[k].y) + (v[k].z + v[k].w);
  mu = group_sum<32>(s) * inv_c;
  float q = 0.0f;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    if (lane + 32 * k < C4) {
      const float a = v[k].x - mu, bb = v[k].y - mu, c = v[k].z - mu, d = v[k].w - mu;
      q += (a * a + bb * bb) + (c * c + d * d);
    }
  }
  rs = rsqrtf(group_sum<32>(q) * inv_c + eps);
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    if (lane + 32 * k < C4)
      out[k] = make_float4((v[k].x - mu) * rs * g[k].x + b[k].x, (v[k].y - mu) * rs * g[k].y + b[k].y,
                           (v[k].z - mu) * rs * g[k].z + b[k].z, (v[k].w - mu) * rs * g[k].w + b[k].w);
    else
      out[k] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

template <int NV>
__device__ __forceinline__ void ln_row(const float* __restrict__ xr, int C4, int lane, float inv_c, float eps,
                                       const float4 (&g)[NV], const float4 (&b)[NV], float4 (&out)[NV],
                                       float& mu, float& rs) {
  float4 v[NV];
  load_row<NV>(xr, C4, lane, v);
  ln_vals<NV>(v, C4, lane, inv_c, eps, g, b, out, mu, rs);
}

__device__ __forceinline__ float silu_f(float u) { return u / (1.0f + expf(-u)); }
// d silu / du = s (1 + u (1 - s)), s = sigmoid(u)
__device__ __forceinline__ float silu_grad(float u) {
  const float s = 1.0f / (1.0f + expf(-u));
  return s * (1.0f + u * (1.0f - s));
}

__device__ __forceinline__ float4 fma4(const float4& a, const float4& b, const float4& c) {
  return make_float4(fmaf(a.x, b.x, c.x), fmaf(a.y, b.y, c.y), fmaf(a.z, b.z, c.z), fmaf(a.w, b.w, c.w));
}

template <int NV, int K>
__global__ void __launch_bounds__(256) lnconv_fwd_kernel(const float* __restrict__ x, const float* __restrict__ lg,
                                                         const float* __restrict__ lb, const float* __restrict__ cw,
                                                         const float* __restrict__ cb, float* __restrict__ y,
                                                         float* __restrict__ mean_out, float* __restrict__ rstd_out,
                                                         int64_t B, int64_t T, int C, int TCH, float eps) {
  const int lane = threadIdx.x & 31;
  const int C4 = C >> 2;
  const float inv_c = 1.0f / (float)C;
  float4 g[NV], lbv[NV], bias[NV], w[K][NV];
  load_row_params<NV>(lg, C4, lane, g);
  load_row_params<NV>(lb, C4, lane, lbv);
  load_row_params<NV>(cb, C4, lane, bias);
  load_conv_taps<NV, K>(cw, C4, lane, w);
  const int64_t nch = (T + TCH - 1) / TCH;
  const int64_t items = B * nch;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t it = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); it < items; it += warps) {
    const int64_t b = it / nch;
    const int64_t t0 = (it % nch) * TCH;
    const int64_t t1 = min(T, t0 + (int64_t)TCH);
    float4 ring[K][NV];  // ring[K - 1] = newest row
#pragma unroll
    for (int q = 0; q < K; ++q)
#pragma unroll
      for (int k = 0; k < NV; ++k) ring[q][k] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int q = 0; q + 1 < K; ++q) {  // rows t0 - K + 1 .. t0 - 1 into ring[1 .. K - 1]
      const int64_t tau = t0 - (K - 1) + q;
      if (tau >= 0) {
        float mu, rs;
        ln_row<NV>(x + (b * T + tau) * C, C4, lane, inv_c, eps, g, lbv, ring[q + 1], mu, rs);
      }
    }
    float4 cur[NV];
    load_row<NV>(x + (b * T + t0) * C, C4, lane, cur);
    for (int64_t t = t0; t < t1; ++t) {
      float4 nxt[NV];  // the next row is in flight while this one is normalised
      if (t + 1 < t1) {
        load_row<NV>(x + (b * T + t + 1) * C, C4, lane, nxt);
      } else {
#pragma unroll
        for (int k = 0; k < NV; ++k) nxt[k] = cur[k];
      }
#pragma unroll
      for (int q = 0; q + 1 < K; ++q)
#pragma unroll
        for (int k = 0; k < NV; ++k) ring[q][k] = ring[q + 1][k];
      float mu, rs;
      const int64_t row = b * T + t;
      ln_vals<NV>(cur, C4, lane, inv_c, eps, g, lbv, ring[K - 1], mu, rs);
#pragma unroll
      for (int k = 0; k < NV; ++k) cur[k] = nxt[k];
      if (lane == 0) {
        mean_out[row] = mu;
        rstd_out[row] = rs;
      }
      float4* yr = reinterpret_cast<float4*>(y + row * C);
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const int jc = lane + 32 * k;
        if (jc < C4) {
          float4 u = bias[k];
#pragma unroll
          for (int j = 0; j < K; ++j) u = fma4(w[j][k], ring[j][k], u);
          yr[jc] = make_float4(silu_f(u.x), silu_f(u.y), silu_f(u.z), silu_f(u.w));
        }
      }
    }
  }
}

template <int NV, int K>
__global__ void __launch_bounds__(256, NV == 1 ? 2 : 1) lnconv_bwd_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                                                         const float* __restrict__ mean, const float* __restrict__ rstd,
                                                         const float* __restrict__ lg, const float* __restrict__ lb,
                                                         const float* __restrict__ cw, const float* __restrict__ cb,
                                                         float* __restrict__ dx, float* __restrict__ part,
                                                         int64_t B, int64_t T, int C, int TCH) {
  __shared__ __align__(16) float red[8][256 + 4];  // rows of 1040 B: float4 stores stay aligned
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int C4 = C >> 2;
  const float inv_c = 1.0f / (float)C;
  float4 g[NV], lbv[NV], bias[NV], w[K][NV];
  load_row_params<NV>(lg, C4, lane, g);
  load_row_params<NV>(lb, C4, lane, lbv);
  load_row_params<NV>(cb, C4, lane, bias);
  load_conv_taps<NV, K>(cw, C4, lane, w);
  const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
  float4 aw[K][NV], acb[NV], ag[NV], ab[NV];
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    acb[k] = ag[k] = ab[k] = z4;
#pragma unroll
    for (int j = 0; j < K; ++j) aw[j][k] = z4;
  }
  const int64_t nch = (T + TCH - 1) / TCH;
  const int64_t items = B * nch;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t it = blockIdx.x * (int64_t)(blockDim.x >> 5) + wid; it < items; it += warps) {
    const int64_t b = it / nch;
    const int64_t t0 = (it % nch) * TCH;
    const int64_t t1 = min(T, t0 + (int64_t)TCH);
    float4 lr[K][NV], dr[K][NV];  // LayerNorm rows and conv-output gradients, [K - 1] = row tau
#pragma unroll
    for (int q = 0; q < K; ++q)
#pragma unroll
      for (int k = 0; k < NV; ++k) lr[q][k] = dr[q][k] = z4;
    auto ln_of = [&](int64_t tau, float4 (&out)[NV]) {  // LayerNorm row from the saved statistics
      const float mu = __ldg(mean + b * T + tau), rs = __ldg(rstd + b * T + tau);
      const float4* xr = reinterpret_cast<const float4*>(x + (b * T + tau) * C);
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const int jc = lane + 32 * k;
        if (jc < C4) {
          const float4 v = __ldg(xr + jc);
          out[k] = make_float4((v.x - mu) * rs * g[k].x + lbv[k].x, (v.y - mu) * rs * g[k].y + lbv[k].y,
                               (v.z - mu) * rs * g[k].z + lbv[k].z, (v.w - mu) * rs * g[k].w + lbv[k].w);
        } else {
          out[k] = z4;
        }
      }
    };
#pragma unroll
    for (int q = 0; q + 1 < K; ++q) {
      const int64_t tau = t0 - (K - 1) + q;
      if (tau >= 0) ln_of(tau, lr[q + 1]);
    }
    // row tau's x, dy and statistics are loaded one iteration ahead
    float4 cx[NV], cdy[NV];
    float cm = 0.0f, cr = 0.0f;
    auto fetch = [&](int64_t tau, float4 (&xv)[NV], float4 (&dv)[NV], float& m, float& r) {
      load_row<NV>(x + (b * T + tau) * C, C4, lane, xv);
      load_row<NV>(dy + (b * T + tau) * C, C4, lane, dv);
      m = __ldg(mean + b * T + tau);
      r = __ldg(rstd + b * T + tau);
    };
    fetch(t0, cx, cdy, cm, cr);
    for (int64_t tau = t0; tau < t1 + (K - 1); ++tau) {
      float4 nx[NV], ndy[NV];
      float nm = 0.0f, nr = 0.0f;
      if (tau + 1 < T && tau + 1 < t1 + (K - 1)) {
        fetch(tau + 1, nx, ndy, nm, nr);
      } else {
#pragma unroll
        for (int k = 0; k < NV; ++k) nx[k] = ndy[k] = z4;
      }
#pragma unroll
      for (int q = 0; q + 1 < K; ++q)
#pragma unroll
        for (int k = 0; k < NV; ++k) {
          lr[q][k] = lr[q + 1][k];
          dr[q][k] = dr[q + 1][k];
        }
      if (tau < T) {
#pragma unroll
        for (int k = 0; k < NV; ++k) {
          const float4 v = cx[k];
          lr[K - 1][k] = lane + 32 * k < C4
                             ? make_float4((v.x - cm) * cr * g[k].x + lbv[k].x, (v.y - cm) * cr * g[k].y + lbv[k].y,
                                           (v.z - cm) * cr * g[k].z + lbv[k].z, (v.w - cm) * cr * g[k].w + lbv[k].w)
                             : z4;
        }
#pragma unroll
        for (int k = 0; k < NV; ++k) {
          const int jc = lane + 32 * k;
          float4 du = z4;
          if (jc < C4) {
            float4 u = bias[k];
#pragma unroll
            for (int j = 0; j < K; ++j) u = fma4(w[j][k], lr[j][k], u);
            const float4 d = cdy[k];
            du = make_float4(d.x * silu_grad(u.x), d.y * silu_grad(u.y), d.z * silu_grad(u.z), d.w * silu_grad(u.w));
          }
          dr[K - 1][k] = du;
          if (tau < t1) {  // this chunk's outputs: conv parameter gradients
            acb[k] = make_float4(acb[k].x + du.x, acb[k].y + du.y, acb[k].z + du.z, acb[k].w + du.w);
#pragma unroll
            for (int j = 0; j < K; ++j) aw[j][k] = fma4(du, lr[j][k], aw[j][k]);
          }
        }
      } else {
#pragma unroll
        for (int k = 0; k < NV; ++k) lr[K - 1][k] = dr[K - 1][k] = z4;
      }
      const int64_t s = tau - (K - 1);  // every du that reaches LayerNorm row s is known now
      if (s >= t0) {
        const int64_t row = b * T + s;
        const float mu = __ldg(mean + row), rs = __ldg(rstd + row);
        const float4* xr = reinterpret_cast<const float4*>(x + row * C);
        float4 xh[NV], wd[NV], dl[NV];
        float s1 = 0.0f, s2 = 0.0f;
#pragma unroll
        for (int k = 0; k < NV; ++k) {
          const int jc = lane + 32 * k;
          float4 d = z4;
#pragma unroll
          for (int j = 0; j < K; ++j) d = fma4(w[j][k], dr[K - 1 - j][k], d);
          dl[k] = d;
          if (jc < C4) {
            const float4 v = __ldg(xr + jc);
            xh[k] = make_float4((v.x - mu) * rs, (v.y - mu) * rs, (v.z - mu) * rs, (v.w - mu) * rs);
          } else {
            xh[k] = z4;
          }
          wd[k] = make_float4(d.x * g[k].x, d.y * g[k].y, d.z * g[k].z, d.w * g[k].w);
          s1 += dot4(wd[k], xh[k]);
          s2 += (wd[k].x + wd[k].y) + (wd[k].z + wd[k].w);
        }
        s1 = group_sum<32>(s1) * inv_c;
        s2 = group_sum<32>(s2) * inv_c;
        float4* o = reinterpret_cast<float4*>(dx + row * C);
#pragma unroll
        for (int k = 0; k < NV; ++k) {
          const int jc = lane + 32 * k;
          if (jc < C4) {
            o[jc] = make_float4((wd[k].x - xh[k].x * s1 - s2) * rs, (wd[k].y - xh[k].y * s1 - s2) * rs,
                                (wd[k].z - xh[k].z * s1 - s2) * rs, (wd[k].w - xh[k].w * s1 - s2) * rs);
            ag[k] = fma4(dl[k], xh[k], ag[k]);
            ab[k] = make_float4(ab[k].x + dl[k].x, ab[k].y + dl[k].y, ab[k].z + dl[k].z, ab[k].w + dl[k].w);
          }
        }
      }
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        cx[k] = nx[k];
        cdy[k] = ndy[k];
      }
      cm = nm;
      cr = nr;
    }
  }
  // per-CTA sums: part[blockIdx.x, q * C + c], q = conv taps 0..K-1, conv bias, ln weight, ln bias
  const int64_t base = (int64_t)blockIdx.x * (K + 3) * C;
#pragma unroll
  for (int q = 0; q < K + 3; ++q) {
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int jc = lane + 32 * k;
      if (jc < C4) {
        const float4 v = q < K ? aw[q < K ? q : 0][k] : (q == K ? acb[k] : (q == K + 1 ? ag[k] : ab[k]));
        *reinterpret_cast<float4*>(&red[wid][4 * jc]) = v;
      }
    }
    __syncthreads();
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
      float t = 0.0f;
#pragma unroll
      for (int v = 0; v < 8; ++v) t += red[v][c];
      part[base + (int64_t)q * C + c] = t;
    }
    __syncthreads();
  }
}

// Sum the per-CTA partials: 32 columns per CTA (deterministic order), scattered to the
// parameter layouts (conv weight [C, 1, K]).
__global__ void __launch_bounds__(256) lnconv_param_reduce_kernel(const float* __restrict__ part, int P, int C, int K,
                                                                  float* __restrict__ dcw, float* __restrict__ dcb,
                                                                  float* __restrict__ dlg, float* __restrict__ dlb) {
  __shared__ float acc[8][33];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int Q = (K + 3) * C;
  const int col = blockIdx.x * 32 + lane;
  float t0 = 0.0f, t1 = 0.0f, t2 = 0.0f, t3 = 0.0f;  // four independent chains
  if (col < Q) {
    int p = wid;
    for (; p + 24 < P; p += 32) {
      t0 += part[(int64_t)p * Q + col];
      t1 += part[(int64_t)(p + 8) * Q + col];
      t2 += part[(int64_t)(p + 16) * Q + col];
      t3 += part[(int64_t)(p + 24) * Q + col];
    }
    for (; p < P; p += 8) t0 += part[(int64_t)p * Q + col];
  }
  acc[wid][lane] = (t0 + t1) + (t2 + t3);
  __syncthreads();
  if (wid == 0 && col < Q) {
    float u = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) u += acc[w][lane];
    const int q = col / C, c = col % C;
    if (q < K) {
      if (dcw) dcw[c * K + q] = u;
    } else if (q == K) {
      if (dcb) dcb[c] = u;
    } else if (q == K + 1) {
      if (dlg) dlg[c] = u;
    } else if (dlb) {
      dlb[c] = u;
    }
  }
}

int lnconv_chunk(int64_t B, int64_t T) {
  // ~148 SMs x 32 warps of work items, 8..64 steps per warp
  const int64_t target = 148 * 32;
  int64_t tc = (B * T + target - 1) / target;
  tc = tc < 8 ? 8 : (tc > 64 ? 64 : tc);
  return (int)tc;
}

unsigned lnconv_grid(int64_t B, int64_t T, int tc) {
  const int64_t items = B * ((T + tc - 1) / tc);
  const int64_t blocks = (items + 7) / 8;
  const int64_t cap = 148 * 4;
  return (unsigned)(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}

int lnconv_check(const char* fn, int64_t B, int64_t T, int C, int K) {
  if (B < 0 || T < 0 || C <= 0 || C % 4 != 0 || C > 256 || K < 1 || K > 4) {
    char buf[200];
    snprintf(buf, sizeof(buf), "%s: needs B, T >= 0, 0 < C <= 256 with C %% 4 == 0 and 1 <= K <= 4", fn);
    return set_error(CSN_ERR_UNSUPPORTED, buf);
  }
  return CSN_OK;
}

template <int NV>
void lnconv_fwd_launch(int K, unsigned grid, cudaStream_t st, const float* x, const float* lg, const float* lb,
                       const float* cw, const float* cb, float* y, float* mean, float* rstd, int64_t B, int64_t T,
                       int C, int tc, float eps) {
  switch (K) {
    case 1: lnconv_fwd_kernel<NV, 1><<<grid, 256, 0, st>>>(x, lg, lb, cw, cb, y, mean, rstd, B, T, C, tc, eps); break;
    case 2: lnconv_fwd_kernel<NV, 2><<<grid, 256, 0, st>>>(x, lg, lb, cw, cb, y, mean, rstd, B, T, C, tc, eps); break;
    case 3: lnconv_fwd_kernel<NV, 3><<<grid, 256, 0, st>>>(x, lg, lb, cw, cb, y, mean, rstd, B, T, C, tc, eps); break;
    default: lnconv_fwd_kernel<NV, 4><<<grid, 256, 0, st>>>(x, lg, lb, cw, cb, y, mean, rstd, B, T, C, tc, eps); break;
  }
}

template <int NV>
void lnconv_bwd_launch(int K, unsigned grid, cudaStream_t st, const float* dy, const float* x, const float* mean,
                       const float* rstd, const float* lg, const float* lb, const float* cw, const float* cb,
                       float* dx, float* part, int64_t B, int64_t T, int C, int tc) {
  switch (K) {
    case 1: lnconv_bwd_kernel<NV, 1><<<grid, 256, 0, st>>>(dy, x, mean, rstd, lg, lb, cw, cb, dx, part, B, T, C, tc); break;
    case 2: lnconv_bwd_kernel<NV, 2><<<grid, 256, 0, st>>>(dy, x, mean, rstd, lg, lb, cw, cb, dx, part, B, T, C, tc); break;
    case 3: lnconv_bwd_kernel<NV, 3><<<grid, 256, 0, st>>>(dy, x, mean, rstd, lg, lb, cw, cb, dx, part, B, T, C, tc); break;
    default: lnconv_bwd_kernel<NV, 4><<<grid, 256, 0, st>>>(dy, x, mean, rstd, lg, lb, cw, cb, dx, part, B, T, C, tc); break;
  }
}

// ------------------------------------------------------------ least-action terms
// V = 4: float4 accesses (R and the head width R / H multiples of 4, 16-byte aligned rows);
// V = 1: scalar.
template <int V>
__device__ __forceinline__ void ldv(const float* p, float (&v)[V]) {
  if constexpr (V == 4) {
    const float4 f = __ldg(reinterpret_cast<const float4*>(p));
    v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
  } else {
    v[0] = __ldg(p);
  }
}

template <int V>
__global__ void __launch_bounds__(256) gen_action_fwd_kernel(const float* __restrict__ biv, const float* __restrict__ dt,
                                                             int64_t B, int64_t T, int R, int H,
                                                             float* __restrict__ part) {
  __shared__ float red[8][2];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int seg = R / H;
  float ak = 0.0f, as = 0.0f;
  const int64_t rows = B * T;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t row = blockIdx.x * (int64_t)(blockDim.x >> 5) + wid; row < rows; row += warps) {
    const bool has_prev = (row % T) != 0;
    for (int j = V * lane; j < R; j += 32 * V) {
      const int h = H == 1 ? 0 : j / seg;
      const float hd = 0.5f * __ldg(dt + row * H + h);
      float bv[V];
      ldv<V>(biv + row * R + j, bv);
      float bp[V];
      float hp = 0.0f;
      if (has_prev) {
        hp = 0.5f * __ldg(dt + (row - 1) * H + h);
        ldv<V>(biv + (row - 1) * R + j, bp);
      }
#pragma unroll
      for (int u = 0; u < V; ++u) {
        const float w = hd * bv[u];
        ak = fmaf(w, w, ak);
        if (has_prev) {
          const float d = w - hp * bp[u];
          as = fmaf(d, d, as);
        }
      }
    }
  }
  ak = group_sum<32>(ak);
  as = group_sum<32>(as);
  if (lane == 0) {
    red[wid][0] = ak;
    red[wid][1] = as;
  }
  __syncthreads();
  if (threadIdx.x < 2) {
    float t = 0.0f;
#pragma unroll
    for (int v = 0; v < 8; ++v) t += red[v][threadIdx.x];
    part[2 * (int64_t)blockIdx.x + threadIdx.x] = t;
  }
}

// out[q] = c[q] * sum_p part[p, q]   (one CTA, fixed order)
__global__ void __launch_bounds__(256) gen_action_finish_kernel(const float* __restrict__ part, int P, float ck,
                                                                float cs, float* __restrict__ out) {
  __shared__ float red[2][256];
  for (int q = 0; q < 2; ++q) {
    float t = 0.0f;
    for (int p = threadIdx.x; p < P; p += blockDim.x) t += part[2 * p + q];
    red[q][threadIdx.x] = t;
  }
  __syncthreads();
  for (int o = 128; o > 0; o >>= 1) {
    if (threadIdx.x < o) {
      red[0][threadIdx.x] += red[0][threadIdx.x + o];
      red[1][threadIdx.x] += red[1][threadIdx.x + o];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    out[0] = ck * red[0][0];
    out[1] = cs * red[1][0];
  }
}

template <int V>
__global__ void __launch_bounds__(256) gen_action_bwd_kernel(const float* __restrict__ biv, const float* __restrict__ dt,
                                                             const float* __restrict__ gk, const float* __restrict__ gs,
                                                             float ck, float cs, int64_t B, int64_t T, int R, int H,
                                                             float* __restrict__ dbiv, float* __restrict__ ddt) {
  const int lane = threadIdx.x & 31;
  const int seg = R / H;
  const float a = 2.0f * ck * (gk ? __ldg(gk) : 0.0f);
  const float c = 2.0f * cs * (gs ? __ldg(gs) : 0.0f);
  const int64_t rows = B * T;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t row = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); row < rows; row += warps) {
    const int64_t t = row % T;
    const bool prev = t > 0, next = t + 1 < T;
    for (int h = 0; h < H; ++h) {
      const float hdt = 0.5f * __ldg(dt + row * H + h);
      const float hdp = prev ? 0.5f * __ldg(dt + (row - 1) * H + h) : 0.0f;
      const float hdn = next ? 0.5f * __ldg(dt + (row + 1) * H + h) : 0.0f;
      float acc = 0.0f;
      for (int j = h * seg + V * lane; j < (h + 1) * seg; j += 32 * V) {
        float bv[V], bp[V], bn[V], out[V];
        ldv<V>(biv + row * R + j, bv);
        if (prev) ldv<V>(biv + (row - 1) * R + j, bp);
        if (next) ldv<V>(biv + (row + 1) * R + j, bn);
#pragma unroll
        for (int u = 0; u < V; ++u) {
          const float w = hdt * bv[u];
          float dw = a * w;
          if (prev) dw = fmaf(c, w - hdp * bp[u], dw);
          if (next) dw = fmaf(-c, hdn * bn[u] - w, dw);
          out[u] = dw * hdt;
          acc = fmaf(dw, 0.5f * bv[u], acc);
        }
        if (dbiv) {
          if constexpr (V == 4) *reinterpret_cast<float4*>(dbiv + row * R + j) = make_float4(out[0], out[1], out[2], out[3]);
          else dbiv[row * R + j] = out[0];
        }
      }
      acc = group_sum<32>(acc);
      if (lane == 0 && ddt) ddt[row * H + h] = acc;
    }
  }
}

bool action_vec4(const float* biv, int R, int H) {
  return R % 4 == 0 && (R / H) % 4 == 0 && (reinterpret_cast<uintptr_t>(biv) & 15u) == 0;
}

unsigned action_grid(int64_t rows) {
  const int64_t blocks = (rows + 7) / 8;
  const int64_t cap = 148 * 8;
  return (unsigned)(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}

// --------------------------------------------------------------- projection epilogue
__device__ __forceinline__ float softplus_f(float x) { return x > 20.0f ? x : log1pf(expf(x)); }
__device__ __forceinline__ float softplus_grad(float x) {
  if (x > 20.0f) return 1.0f;
  const float z = expf(x);
  return z / (z + 1.0f);
}

// One warp per row: lanes walk the row's columns (coalesced).
__global__ void __launch_bounds__(256) proj_epilogue_fwd_kernel(const float* __restrict__ raw, int64_t R, int N, int K,
                                                                int HT, const float* __restrict__ scale, float dt_base,
                                                                float* __restrict__ biv, float* __restrict__ gamma,
                                                                float* __restrict__ dt) {
  const int lane = threadIdx.x & 31;
  const int NK = N * K, Q = NK + N + HT;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); r < R; r += warps) {
    const float* rr = raw + r * Q;
    for (int c = lane; c < NK; c += 32) biv[r * NK + c] = __ldg(rr + c) * __ldg(scale + c / K);
    for (int c = lane; c < N; c += 32) gamma[r * N + c] = softplus_f(__ldg(rr + NK + c));
    for (int c = lane; c < HT; c += 32) dt[r * HT + c] = softplus_f(__ldg(rr + NK + N + c)) * dt_base;
  }
}

// One warp per row: the gradient row elementwise (coalesced), then lane n sums neuron n's
// K products for part[r, n] (the row is in L1 by then).
__global__ void __launch_bounds__(256) proj_epilogue_bwd_kernel(const float* __restrict__ raw, int64_t R, int N, int K,
                                                                int HT, const float* __restrict__ scale, float dt_base,
                                                                const float* __restrict__ dbiv,
                                                                const float* __restrict__ dgamma,
                                                                const float* __restrict__ ddt, float* __restrict__ draw,
                                                                float* __restrict__ part) {
  const int lane = threadIdx.x & 31;
  const int NK = N * K, Q = NK + N + HT;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); r < R; r += warps) {
    const float* rr = raw + r * Q;
    float* dr = draw + r * Q;
    for (int c = lane; c < NK; c += 32) dr[c] = (dbiv ? __ldg(dbiv + r * NK + c) : 0.0f) * __ldg(scale + c / K);
    for (int c = lane; c < N; c += 32)
      dr[NK + c] = (dgamma ? __ldg(dgamma + r * N + c) : 0.0f) * softplus_grad(__ldg(rr + NK + c));
    for (int c = lane; c < HT; c += 32)
      dr[NK + N + c] = (ddt ? __ldg(ddt + r * HT + c) : 0.0f) * dt_base * softplus_grad(__ldg(rr + NK + N + c));
    for (int n = lane; n < N; n += 32) {
      float acc = 0.0f;
      if (dbiv)
        for (int k = 0; k < K; ++k) acc = fmaf(__ldg(dbiv + r * NK + n * K + k), __ldg(rr + n * K + k), acc);
      part[r * N + n] = acc;
    }
  }
}

// ------------------------------------------------------------------- column sum
// part[cta, c] = sum over this CTA's rows (contiguous row range); 256 threads over columns.
__global__ void __launch_bounds__(256) colsum_partial_kernel(const float* __restrict__ x, int64_t R, int C, int64_t rows_per,
                                                             float* __restrict__ part) {
  const int64_t r0 = blockIdx.x * rows_per;
  const int64_t r1 = min(R, r0 + rows_per);
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    float t0 = 0.0f, t1 = 0.0f, t2 = 0.0f, t3 = 0.0f;
    int64_t r = r0;
    for (; r + 3 < r1; r += 4) {
      t0 += __ldg(x + r * C + c);
      t1 += __ldg(x + (r + 1) * C + c);
      t2 += __ldg(x + (r + 2) * C + c);
      t3 += __ldg(x + (r + 3) * C + c);
    }
    for (; r < r1; ++r) t0 += __ldg(x + r * C + c);
    part[(int64_t)blockIdx.x * C + c] = (t0 + t1) + (t2 + t3);
  }
}

// out[c] = sum_p part[p, c]: 32 columns per CTA, 8 warps over interleaved rows, fixed order.
__global__ void __launch_bounds__(256) colsum_finish_kernel(const float* __restrict__ part, int P, int C,
                                                            float* __restrict__ out) {
  __shared__ float acc[8][33];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + lane;
  float t0 = 0.0f, t1 = 0.0f;
  if (c < C) {
    int p = wid;
    for (; p + 8 < P; p += 16) {
      t0 += part[(int64_t)p * C + c];
      t1 += part[(int64_t)(p + 8) * C + c];
    }
    for (; p < P; p += 8) t0 += part[(int64_t)p * C + c];
  }
  acc[wid][lane] = t0 + t1;
  __syncthreads();
  if (wid == 0 && c < C) {
    float u = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) u += acc[w][lane];
    out[c] = u;
  }
}

void colsum_plan(int64_t R, int64_t& ctas, int64_t& rows_per) {
  const int64_t target = 148 * 4;
  rows_per = (R + target - 1) / target;
  if (rows_per < 16) rows_per = 16;
  ctas = (R + rows_per - 1) / rows_per;
  if (ctas < 1) ctas = 1;
}

// ------------------------------------------------------------------------ gate
// One warp per row; V = 4: float4 columns (F % 4 == 0, 16-byte aligned rows).
template <int V>
__device__ __forceinline__ void ld_v(const float* p, float (&v)[V]) {
  if constexpr (V == 4) {
    const float4 f = __ldg(reinterpret_cast<const float4*>(p));
    v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
  } else {
    v[0] = __ldg(p);
  }
}
template <int V>
__device__ __forceinline__ void st_v(float* p, const float (&v)[V]) {
  if constexpr (V == 4) *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  else p[0] = v[0];
}

template <int V>
__global__ void __launch_bounds__(256) silu_gate_fwd_kernel(const float* __restrict__ gu, int64_t R, int F,
                                                            float* __restrict__ y) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); r < R; r += warps) {
    const float* g0 = gu + r * 2 * F;
    for (int f = V * lane; f < F; f += 32 * V) {
      float g[V], u[V], o[V];
      ld_v<V>(g0 + f, g);
      ld_v<V>(g0 + F + f, u);
#pragma unroll
      for (int q = 0; q < V; ++q) o[q] = silu_f(g[q]) * u[q];
      st_v<V>(y + r * F + f, o);
    }
  }
}

template <int V>
__global__ void __launch_bounds__(256) silu_gate_bwd_kernel(const float* __restrict__ gu, const float* __restrict__ dy,
                                                            int64_t R, int F, float* __restrict__ dgu) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); r < R; r += warps) {
    const float* g0 = gu + r * 2 * F;
    float* d0 = dgu + r * 2 * F;
    for (int f = V * lane; f < F; f += 32 * V) {
      float g[V], u[V], d[V], dg[V], du[V];
      ld_v<V>(g0 + f, g);
      ld_v<V>(g0 + F + f, u);
      ld_v<V>(dy + r * F + f, d);
#pragma unroll
      for (int q = 0; q < V; ++q) {
        dg[q] = d[q] * u[q] * silu_grad(g[q]);
        du[q] = d[q] * silu_f(g[q]);
      }
      st_v<V>(d0 + f, dg);
      st_v<V>(d0 + F + f, du);
    }
  }
}

bool gate_vec4(const void* a, const void* b, const void* c, int F) {
  const uintptr_t m = reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
                      reinterpret_cast<uintptr_t>(c);
  return F % 4 == 0 && (m & 15u) == 0;
}

unsigned row_grid(int64_t rows) {  // warp per row, 8 warps per CTA
  const int64_t blocks = (rows + 7) / 8;
  const int64_t cap = 148 * 16;
  return (unsigned)(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
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

extern "C" int csn_ln_conv_silu_fwd(const float* x, const float* ln_weight, const float* ln_bias,
                                    const float* conv_weight, const float* conv_bias, float* y, float* mean,
                                    float* rstd, int64_t B, int64_t T, int C, int K, float eps, void* stream) {
  if (int rc = lnconv_check("csn_ln_conv_silu_fwd", B, T, C, K)) return rc;
  if (B * T == 0) return CSN_OK;
  if (!x || !ln_weight || !ln_bias || !conv_weight || !conv_bias || !y || !mean || !rstd || !al16(x) || !al16(y) ||
      !al16(ln_weight) || !al16(ln_bias) || !al16(conv_bias))
    return set_error(CSN_ERR_INVALID, "csn_ln_conv_silu_fwd: missing or misaligned pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int tc = lnconv_chunk(B, T);
  const unsigned grid = lnconv_grid(B, T, tc);
  KernelTimer kt("ln_conv_silu_fwd", st);
  if (C <= 128)
    lnconv_fwd_launch<1>(K, grid, st, x, ln_weight, ln_bias, conv_weight, conv_bias, y, mean, rstd, B, T, C, tc, eps);
  else
    lnconv_fwd_launch<2>(K, grid, st, x, ln_weight, ln_bias, conv_weight, conv_bias, y, mean, rstd, B, T, C, tc, eps);
  return check_launch("csn_ln_conv_silu_fwd");
}

extern "C" size_t csn_ln_conv_silu_bwd_workspace_bytes(int64_t B, int64_t T, int C, int K) {
  if (B <= 0 || T <= 0 || C <= 0 || K <= 0) return 0;
  return (size_t)lnconv_grid(B, T, lnconv_chunk(B, T)) * (size_t)(K + 3) * (size_t)C * sizeof(float);
}

extern "C" int csn_ln_conv_silu_bwd(const float* dy, const float* x, const float* mean, const float* rstd,
                                    const float* ln_weight, const float* ln_bias, const float* conv_weight,
                                    const float* conv_bias, float* dx, float* dln_weight, float* dln_bias,
                                    float* dconv_weight, float* dconv_bias, int64_t B, int64_t T, int C, int K,
                                    void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = lnconv_check("csn_ln_conv_silu_bwd", B, T, C, K)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (B * T == 0) {
    float* outs[4] = {dln_weight, dln_bias, dconv_weight, dconv_bias};
    const size_t n[4] = {(size_t)C, (size_t)C, (size_t)C * K, (size_t)C};
    for (int i = 0; i < 4; ++i)
      if (outs[i] && cudaMemsetAsync(outs[i], 0, n[i] * sizeof(float), st) != cudaSuccess)
        return set_error(CSN_ERR_CUDA, "csn_ln_conv_silu_bwd: cudaMemsetAsync");
    return CSN_OK;
  }
  if (!dy || !x || !mean || !rstd || !ln_weight || !ln_bias || !conv_weight || !conv_bias || !dx || !al16(dy) ||
      !al16(x) || !al16(dx) || !al16(ln_weight) || !al16(ln_bias) || !al16(conv_bias))
    return set_error(CSN_ERR_INVALID, "csn_ln_conv_silu_bwd: missing or misaligned pointer");
  const int tc = lnconv_chunk(B, T);
  const unsigned grid = lnconv_grid(B, T, tc);
  if (!workspace || workspace_bytes < csn_ln_conv_silu_bwd_workspace_bytes(B, T, C, K))
    return set_error(CSN_ERR_INVALID,
                     "csn_ln_conv_silu_bwd: workspace smaller than csn_ln_conv_silu_bwd_workspace_bytes");
  float* part = static_cast<float*>(workspace);
  {
    KernelTimer kt("ln_conv_silu_bwd", st);
    if (C <= 128)
      lnconv_bwd_launch<1>(K, grid, st, dy, x, mean, rstd, ln_weight, ln_bias, conv_weight, conv_bias, dx, part, B,
                           T, C, tc);
    else
      lnconv_bwd_launch<2>(K, grid, st, dy, x, mean, rstd, ln_weight, ln_bias, conv_weight, conv_bias, dx, part, B,
                           T, C, tc);
  }
  {
    KernelTimer kt("ln_conv_silu_param_reduce", st);
    lnconv_param_reduce_kernel<<<(unsigned)(((K + 3) * C + 31) / 32), 256, 0, st>>>(
        part, (int)grid, C, K, dconv_weight, dconv_bias, dln_weight, dln_bias);
  }
  return check_launch("csn_ln_conv_silu_bwd");
}

extern "C" size_t csn_generator_action_workspace_bytes(int64_t B, int64_t T) {
  return (size_t)action_grid(B * T) * 2 * sizeof(float);
}

extern "C" int csn_generator_action_fwd(const float* biv, const float* dt, int64_t B, int64_t T, int R, int H,
                                        float c_kin, float c_smooth, float* out, void* workspace,
                                        size_t workspace_bytes, void* stream) {
  if (B < 0 || T < 0 || R < 0 || H < 1 || (R % H) != 0)
    return set_error(CSN_ERR_INVALID, "csn_generator_action_fwd: needs B, T, R >= 0, H >= 1 and R % H == 0");
  if (!out) return set_error(CSN_ERR_INVALID, "csn_generator_action_fwd: out is required");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (B * T * R == 0) {
    if (cudaMemsetAsync(out, 0, 2 * sizeof(float), st) != cudaSuccess)
      return set_error(CSN_ERR_CUDA, "csn_generator_action_fwd: cudaMemsetAsync");
    return CSN_OK;
  }
  if (!biv || !dt) return set_error(CSN_ERR_INVALID, "csn_generator_action_fwd: biv and dt are required");
  const unsigned grid = action_grid(B * T);
  if (!workspace || workspace_bytes < csn_generator_action_workspace_bytes(B, T))
    return set_error(CSN_ERR_INVALID, "csn_generator_action_fwd: workspace smaller than csn_generator_action_workspace_bytes");
  float* part = static_cast<float*>(workspace);
  KernelTimer kt("generator_action_fwd", st);
  if (action_vec4(biv, R, H)) gen_action_fwd_kernel<4><<<grid, 256, 0, st>>>(biv, dt, B, T, R, H, part);
  else gen_action_fwd_kernel<1><<<grid, 256, 0, st>>>(biv, dt, B, T, R, H, part);
  gen_action_finish_kernel<<<1, 256, 0, st>>>(part, (int)grid, c_kin, c_smooth, out);
  return check_launch("csn_generator_action_fwd");
}

extern "C" int csn_generator_action_bwd(const float* biv, const float* dt, const float* g_kin, const float* g_smooth,
                                        int64_t B, int64_t T, int R, int H, float c_kin, float c_smooth,
                                        float* dbiv, float* ddt, void* stream) {
  if (B < 0 || T < 0 || R < 0 || H < 1 || (R % H) != 0)
    return set_error(CSN_ERR_INVALID, "csn_generator_action_bwd: needs B, T, R >= 0, H >= 1 and R % H == 0");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (B * T == 0) return CSN_OK;
  if (R == 0) {
    if (ddt && cudaMemsetAsync(ddt, 0, sizeof(float) * B * T * H, st) != cudaSuccess)
      return set_error(CSN_ERR_CUDA, "csn_generator_action_bwd: cudaMemsetAsync");
    return CSN_OK;
  }
  if (!biv || !dt) return set_error(CSN_ERR_INVALID, "csn_generator_action_bwd: biv and dt are required");
  KernelTimer kt("generator_action_bwd", st);
  if (action_vec4(biv, R, H) && (!dbiv || al16(dbiv)))
    gen_action_bwd_kernel<4><<<action_grid(B * T), 256, 0, st>>>(biv, dt, g_kin, g_smooth, c_kin, c_smooth, B, T, R,
                                                                 H, dbiv, ddt);
  else
    gen_action_bwd_kernel<1><<<action_grid(B * T), 256, 0, st>>>(biv, dt, g_kin, g_smooth, c_kin, c_smooth, B, T, R,
                                                                 H, dbiv, ddt);
  return check_launch("csn_generator_action_bwd");
}

extern "C" int csn_projection_epilogue_fwd(const float* raw, int64_t R, int N, int K, int HT,
                                           const float* omega_scale, float dt_base, float* biv, float* gamma,
                                           float* dt, void* stream) {
  if (R < 0 || N < 0 || K < 0 || HT < 0) return set_error(CSN_ERR_INVALID, "csn_projection_epilogue_fwd: negative size");
  const int64_t Q = (int64_t)N * K + N + HT;
  if (R * Q == 0) return CSN_OK;
  if (!raw || (N * K > 0 && (!omega_scale || !biv)) || (N > 0 && !gamma) || (HT > 0 && !dt))
    return set_error(CSN_ERR_INVALID, "csn_projection_epilogue_fwd: missing pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  KernelTimer kt("projection_epilogue_fwd", st);
  proj_epilogue_fwd_kernel<<<row_grid(R), 256, 0, st>>>(raw, R, N, K, HT, omega_scale, dt_base, biv, gamma, dt);
  return check_launch("csn_projection_epilogue_fwd");
}

extern "C" int csn_projection_epilogue_bwd(const float* raw, int64_t R, int N, int K, int HT,
                                           const float* omega_scale, float dt_base, const float* dbiv,
                                           const float* dgamma, const float* ddt, float* draw, float* scale_part,
                                           void* stream) {
  if (R < 0 || N < 0 || K < 0 || HT < 0) return set_error(CSN_ERR_INVALID, "csn_projection_epilogue_bwd: negative size");
  const int64_t J = (int64_t)N + HT;
  if (R * J == 0) return CSN_OK;
  if (!raw || !draw || (N > 0 && (!omega_scale || !scale_part)))
    return set_error(CSN_ERR_INVALID, "csn_projection_epilogue_bwd: missing pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  KernelTimer kt("projection_epilogue_bwd", st);
  proj_epilogue_bwd_kernel<<<row_grid(R), 256, 0, st>>>(raw, R, N, K, HT, omega_scale, dt_base, dbiv, dgamma, ddt,
                                                          draw, scale_part);
  return check_launch("csn_projection_epilogue_bwd");
}

extern "C" size_t csn_column_sum_workspace_bytes(int64_t R, int C) {
  if (R <= 0 || C <= 0) return 0;
  int64_t ctas, rows_per;
  colsum_plan(R, ctas, rows_per);
  return (size_t)ctas * (size_t)C * sizeof(float);
}

extern "C" int csn_column_sum(const float* x, int64_t R, int C, float* out, void* workspace, size_t workspace_bytes,
                              void* stream) {
  if (R < 0 || C < 0) return set_error(CSN_ERR_INVALID, "csn_column_sum: negative size");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (C == 0) return CSN_OK;
  if (!out) return set_error(CSN_ERR_INVALID, "csn_column_sum: out is required");
  if (R == 0) {
    if (cudaMemsetAsync(out, 0, sizeof(float) * C, st) != cudaSuccess)
      return set_error(CSN_ERR_CUDA, "csn_column_sum: cudaMemsetAsync");
    return CSN_OK;
  }
  if (!x) return set_error(CSN_ERR_INVALID, "csn_column_sum: x is required");
  int64_t ctas, rows_per;
  colsum_plan(R, ctas, rows_per);
  if (!workspace || workspace_bytes < csn_column_sum_workspace_bytes(R, C))
    return set_error(CSN_ERR_INVALID, "csn_column_sum: workspace smaller than csn_column_sum_workspace_bytes");
  float* part = static_cast<float*>(workspace);
  KernelTimer kt("column_sum", st);
  colsum_partial_kernel<<<(unsigned)ctas, 256, 0, st>>>(x, R, C, rows_per, part);
  colsum_finish_kernel<<<(unsigned)((C + 31) / 32), 256, 0, st>>>(part, (int)ctas, C, out);
  return check_launch("csn_column_sum");
}

extern "C" int csn_silu_gate_fwd(const float* gu, int64_t R, int F, float* y, void* stream) {
  if (R < 0 || F < 0) return set_error(CSN_ERR_INVALID, "csn_silu_gate_fwd: negative size");
  if (R * F == 0) return CSN_OK;
  if (!gu || !y) return set_error(CSN_ERR_INVALID, "csn_silu_gate_fwd: missing pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  KernelTimer kt("silu_gate_fwd", st);
  if (gate_vec4(gu, y, y, F)) silu_gate_fwd_kernel<4><<<row_grid(R), 256, 0, st>>>(gu, R, F, y);
  else silu_gate_fwd_kernel<1><<<row_grid(R), 256, 0, st>>>(gu, R, F, y);
  return check_launch("csn_silu_gate_fwd");
}

extern "C" int csn_silu_gate_bwd(const float* gu, const float* dy, int64_t R, int F, float* dgu, void* stream) {
  if (R < 0 || F < 0) return set_error(CSN_ERR_INVALID, "csn_silu_gate_bwd: negative size");
  if (R * F == 0) return CSN_OK;
  if (!gu || !dy || !dgu) return set_error(CSN_ERR_INVALID, "csn_silu_gate_bwd: missing pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  KernelTimer kt("silu_gate_bwd", st);
  if (gate_vec4(gu, dy, dgu, F)) silu_gate_bwd_kernel<4><<<row_grid(R), 256, 0, st>>>(gu, dy, R, F, dgu);
  else silu_gate_bwd_kernel<1><<<row_grid(R), 256, 0, st>>>(gu, dy, R, F, dgu);
  return check_launch("csn_silu_gate_bwd");
}
