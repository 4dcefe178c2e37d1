// csn_spatial.cu -- the spatial rotor blocks' generator chain, fused (forward and adjoint).
//
// Per pixel p = (h, w) of image b and neuron n, from the three convolution outputs in NCHW
// (csn_toolkit/csn/vision.py:79-94 for Cl(4), :136-151 for Cl(8)):
//   ds     = softplus(metric[b, n, p])
//   C      = in_proj[b, n*D*D + (i, j), p]                       (D x D injection)
//   skew   = triu scatter of biv_proj[b, n*K + k, p], k row-major over u < v, minus its transpose
//   Omega  = clamp((skew + tanh(lambda) 0.5 (C - C^T)) 0.5 ds, -3, 3)
//   decay  = sigmoid(-softplus(gamma_log[n]) ds)
// The outputs are pixel-major, the layout of the spatial scan: Omega, C [B, H*W, N, D, D] and
// decay [B, H*W, N].  The exact Cayley rotor of Omega and M = decay Q stay separate ops.
// One CTA takes TP pixels of one image: it stages the TP columns of the three NCHW inputs in
// shared memory (reads coalesced along pixels), then writes the pixel-major outputs
// contiguously.  This replaces the permute copies, the zero-filled skew with its two
// index_put scatters, and the eight elementwise ops of the reference chain (and their
// autograd) with one kernel each way.
//
// Adjoint, given dOmega, dC (the scan's gradient of C) and ddecay:
//   g      = dOmega [-3 <= Omega_pre <= 3]         (clamp passes the gradient at the bounds)
//   dpre   = g 0.5 ds
//   dbiv_k = dpre[u][v] - dpre[v][u]
//   dC_in  = dC + 0.5 tanh(lambda) (dpre - dpre^T)
//   dds    = sum_ij g pre 0.5 - ddecay decay (1 - decay) softplus(gamma)
//   dmetric = dds softplus'(metric)
//   dtanh  = sum dpre 0.5 (C - C^T)    -> dlambda = (1 - tanh^2) sum dtanh
//   dgamma = sum -ddecay decay (1 - decay) ds softplus'(gamma)
// dlambda and dgamma are summed per CTA here (fixed order) and over CTAs by the caller.
#include <cstdint>
#include <cstdio>

#include "csn_internal.h"

namespace csn {
namespace {

constexpr int SP_THREADS = 256;
constexpr unsigned SP_FULL = 0xffffffffu;
constexpr int SP_BATCH = 4;      // global loads in flight per thread in the backward's entry loops

// torch.nn.functional.softplus (beta 1, threshold 20) and its derivative
__device__ __forceinline__ float sp_softplus(float x) { return x > 20.0f ? x : log1pf(expf(x)); }
__device__ __forceinline__ float sp_softplus_grad(float x) { return x > 20.0f ? 1.0f : 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float sp_sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }

// generator index of the pair (u, v), u < v, in the row-major upper triangle of D x D
template <int D>
__device__ __forceinline__ int sp_triu_index(int u, int v) { return u * D - u * (u + 1) / 2 + (v - u - 1); }

template <int D>
__device__ __forceinline__ void sp_triu_pair(int k, int& u, int& v) {
  u = 0;
  while (k >= D - 1 - u) {
    k -= D - 1 - u;
    ++u;
  }
  v = u + 1 + k;
}

// pixels per CTA: about 4 K matrix entries per CTA of 256 threads (64 for D = 4, 16 for D = 16)
__host__ __device__ constexpr int sp_tp(int D) { return D == 4 ? 64 : (D == 8 ? 32 : 16); }

// The entries e = threadIdx.x + SP_THREADS m of a CTA's tile as (pixel, entry) = divmod(e, per),
// advanced without dividing (one division per thread at the start)
struct SpIter {
  int pl, r, dq, dr, per;
  __device__ explicit SpIter(int per_) : per(per_) {
    pl = threadIdx.x / per;
    r = threadIdx.x % per;
    dq = SP_THREADS / per;
    dr = SP_THREADS % per;
  }
  __device__ void next() {
    pl += dq;
    r += dr;
    if (r >= per) {
      r -= per;
      ++pl;
    }
  }
};

// Shared-memory tile of one CTA: the NCHW inputs of TP pixels, columns padded to TP + 1.
template <int D>
struct SpTile {
  static constexpr int DD = D * D;
  static constexpr int K = D * (D - 1) / 2;
  static constexpr int TP = sp_tp(D);
  static constexpr int LD = TP + 1;
};

// Tile row of the injection entry (i, j): for D = 16, j is XOR-swizzled by i >> 1, so that a
// warp reading entries (j, i) over j (the transposed read) touches 16 banks instead of 2
// (rows 16 x LD floats apart share a bank pair); D = 4, 8 keep i D + j
template <int D>
__host__ __device__ __forceinline__ int sp_crow(int i, int j) { return D == 16 ? i * D + (j ^ (i >> 1)) : i * D + j; }

// Stage rows [0, rows) of a [B, rows, HW] tensor's TP pixel columns starting at p0 into tile
// rows row_of(r): SP_STAGE loads in flight per thread before their shared-memory stores
constexpr int SP_STAGE = 8;

template <int TP, typename RowOf>
__device__ __forceinline__ void sp_stage_rows(float* dst, const float* __restrict__ src, int rows, int64_t HW,
                                              int64_t b, int64_t p0, int np, RowOf row_of) {
  const int total = rows * TP;
  for (int t0 = threadIdx.x; t0 < total; t0 += SP_THREADS * SP_STAGE) {
    float v[SP_STAGE];
#pragma unroll
    for (int u = 0; u < SP_STAGE; ++u) {
      const int t = t0 + u * SP_THREADS, r = t / TP, pl = t % TP;
      v[u] = (t < total && pl < np) ? __ldg(src + (b * rows + r) * HW + p0 + pl) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < SP_STAGE; ++u) {
      const int t = t0 + u * SP_THREADS;
      if (t < total) dst[row_of(t / TP) * (TP + 1) + t % TP] = v[u];
    }
  }
}

// the NCHW injection columns, into the swizzled tile rows of sp_crow
template <int D, int TP>
__device__ __forceinline__ void sp_stage_c(float* dst, const float* __restrict__ src, int rows, int64_t HW,
                                           int64_t b, int64_t p0, int np) {
  sp_stage_rows<TP>(dst, src, rows, HW, b, p0, np, [](int r) {
    const int ij = r % (D * D);
    return r - ij + sp_crow<D>(ij / D, ij % D);
  });
}

template <int TP>
__device__ __forceinline__ void sp_stage(float* dst, const float* __restrict__ src, int rows, int64_t HW,
                                         int64_t b, int64_t p0, int np) {
  sp_stage_rows<TP>(dst, src, rows, HW, b, p0, np, [](int r) { return r; });
}

// skew + tl 0.5 (C - C^T) at entry (i, j) of neuron n, pixel pl (Omega before the 0.5 ds
// scale and the clamp); J returns 0.5 (C - C^T) there
template <int D>
__device__ __forceinline__ float sp_pre(const float* sC, const float* sB, int n, int i, int j, int pl, float tl,
                                        float& J) {
  using T = SpTile<D>;
  const float cij = sC[(n * T::DD + sp_crow<D>(i, j)) * T::LD + pl];
  const float cji = sC[(n * T::DD + sp_crow<D>(j, i)) * T::LD + pl];
  J = 0.5f * (cij - cji);
  float skew = 0.0f;
  if (i < j) skew = sB[(n * T::K + sp_triu_index<D>(i, j)) * T::LD + pl];
  else if (i > j) skew = -sB[(n * T::K + sp_triu_index<D>(j, i)) * T::LD + pl];
  return skew + tl * J;
}

template <int D>
__global__ void __launch_bounds__(SP_THREADS) spatial_gen_fwd_kernel(
    const float* __restrict__ craw, const float* __restrict__ braw, const float* __restrict__ mraw,
    const float* __restrict__ lambda_sw, const float* __restrict__ gamma_log, float* __restrict__ omega,
    float* __restrict__ cout, float* __restrict__ decay, int64_t HW, int N) {
  using T = SpTile<D>;
  extern __shared__ float sp_smem[];
  float* sC = sp_smem;                          // [N*DD][LD]
  float* sB = sC + N * T::DD * T::LD;           // [N*K][LD]
  float* sM = sB + N * T::K * T::LD;            // [N][LD]  ds
  const int64_t b = blockIdx.y;
  const int64_t p0 = (int64_t)blockIdx.x * T::TP;
  const int np = HW - p0 < T::TP ? (int)(HW - p0) : T::TP;
  sp_stage_c<D, T::TP>(sC, craw, N * T::DD, HW, b, p0, np);
  sp_stage<T::TP>(sB, braw, N * T::K, HW, b, p0, np);
  sp_stage<T::TP>(sM, mraw, N, HW, b, p0, np);
  __syncthreads();
  for (int t = threadIdx.x; t < N * T::TP; t += SP_THREADS) {  // ds = softplus(metric)
    const int n = t / T::TP, pl = t % T::TP;
    sM[n * T::LD + pl] = sp_softplus(sM[n * T::LD + pl]);
  }
  __syncthreads();
  const float tl = tanhf(__ldg(lambda_sw));
  const int per_px = N * T::DD;
  const int64_t base = (b * HW + p0) * per_px;  // first output entry of this CTA
  for (SpIter it(per_px); it.pl < np; it.next()) {
    const int pl = it.pl, r = it.r, e = pl * per_px + r;
    const int n = r / T::DD, ij = r % T::DD, i = ij / D, j = ij % D;
    const float ds = sM[n * T::LD + pl];
    float J;
    const float pre = sp_pre<D>(sC, sB, n, i, j, pl, tl, J);
    omega[base + e] = fminf(fmaxf(pre * (0.5f * ds), -3.0f), 3.0f);
    cout[base + e] = sC[(n * T::DD + sp_crow<D>(i, j)) * T::LD + pl];
    if (ij == 0) {
      const float sg = sp_softplus(__ldg(gamma_log + n));
      decay[(b * HW + p0 + pl) * N + n] = sp_sigmoid(-sg * ds);
    }
  }
}

template <int D>
__global__ void __launch_bounds__(SP_THREADS) spatial_gen_bwd_kernel(
    const float* __restrict__ craw, const float* __restrict__ braw, const float* __restrict__ mraw,
    const float* __restrict__ lambda_sw, const float* __restrict__ gamma_log, const float* __restrict__ d_omega,
    const float* __restrict__ d_c, const float* __restrict__ d_decay, float* __restrict__ dcraw,
    float* __restrict__ dbraw, float* __restrict__ dmraw, float* __restrict__ dlam_part,
    float* __restrict__ dgam_part, int64_t HW, int N) {
  using T = SpTile<D>;
  extern __shared__ float sp_smem[];
  const int per_px = N * T::DD;
  const int LG = per_px + 1;                    // row stride of the pixel-major g tile
  float* sC = sp_smem;                          // [N*DD][LD]; reused for the dC_in tile
  float* sB = sC + N * T::DD * T::LD;           // [N*K][LD]
  float* sRaw = sB + N * T::K * T::LD;          // [N][LD]  metric before softplus
  float* sDs = sRaw + N * T::LD;                // [N][LD]  ds
  float* sDm = sDs + N * T::LD;                 // [N][LD]  dmetric
  float* sG = sDm + N * T::LD;                  // [TP][LG] masked dOmega
  float* sTl = sG + T::TP * LG;                 // [TP*N]
  float* sGam = sTl + T::TP * N;                // [TP*N]
  const int64_t b = blockIdx.y;
  const int64_t p0 = (int64_t)blockIdx.x * T::TP;
  const int np = HW - p0 < T::TP ? (int)(HW - p0) : T::TP;
  const int64_t cta = (int64_t)blockIdx.y * gridDim.x + blockIdx.x;
  __shared__ unsigned char sPair[2][T::K];  // (u, v) of generator k
  for (int k = threadIdx.x; k < T::K; k += SP_THREADS) {
    int u, v;
    sp_triu_pair<D>(k, u, v);
    sPair[0][k] = (unsigned char)u;
    sPair[1][k] = (unsigned char)v;
  }
  sp_stage_c<D, T::TP>(sC, craw, N * T::DD, HW, b, p0, np);
  sp_stage<T::TP>(sB, braw, N * T::K, HW, b, p0, np);
  sp_stage<T::TP>(sRaw, mraw, N, HW, b, p0, np);
  __syncthreads();
  for (int t = threadIdx.x; t < N * T::TP; t += SP_THREADS) {
    const int n = t / T::TP, pl = t % T::TP;
    sDs[n * T::LD + pl] = sp_softplus(sRaw[n * T::LD + pl]);
  }
  __syncthreads();
  const float tl = tanhf(__ldg(lambda_sw));
  const int64_t base = (b * HW + p0) * per_px;
  // 1. g = dOmega where the clamp passed Omega through (SP_BATCH loads in flight per thread)
  for (SpIter it(per_px); it.pl < np;) {
    int pls[SP_BATCH], rs[SP_BATCH];
    float dv[SP_BATCH];
#pragma unroll
    for (int u = 0; u < SP_BATCH; ++u) {
      pls[u] = it.pl;
      rs[u] = it.r;
      dv[u] = it.pl < np ? __ldg(d_omega + base + it.pl * per_px + it.r) : 0.0f;
      it.next();
    }
#pragma unroll
    for (int u = 0; u < SP_BATCH; ++u) {
      const int pl = pls[u], r = rs[u];
      if (pl >= np) break;
      const int n = r / T::DD, ij = r % T::DD, i = ij / D, j = ij % D;
      float J;
      const float om = sp_pre<D>(sC, sB, n, i, j, pl, tl, J) * (0.5f * sDs[n * T::LD + pl]);
      const bool pass = om >= -3.0f && om <= 3.0f;
      sG[pl * LG + r] = pass ? dv[u] : 0.0f;
    }
  }
  __syncthreads();
  // 2. per (pixel, neuron): dds, dmetric and the lambda / gamma contributions (warp sums)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int q = warp; q < np * N; q += SP_THREADS / 32) {
    const int pl = q / N, n = q % N;
    const float ds = sDs[n * T::LD + pl];
    float a = 0.0f, c = 0.0f;
    for (int ij = lane; ij < T::DD; ij += 32) {
      float J;
      const float pre = sp_pre<D>(sC, sB, n, ij / D, ij % D, pl, tl, J);
      const float g = sG[pl * LG + n * T::DD + ij];
      a = fmaf(g * pre, 0.5f, a);
      c = fmaf(g * (0.5f * ds), J, c);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      a += __shfl_xor_sync(SP_FULL, a, o);
      c += __shfl_xor_sync(SP_FULL, c, o);
    }
    if (lane == 0) {
      const float gam = __ldg(gamma_log + n);
      const float sg = sp_softplus(gam);
      const float dec = sp_sigmoid(-sg * ds);
      const float dd = __ldg(d_decay + (b * HW + p0 + pl) * N + n) * dec * (1.0f - dec);
      sDm[n * T::LD + pl] = (a - dd * sg) * sp_softplus_grad(sRaw[n * T::LD + pl]);
      sTl[q] = c;
      sGam[q] = -dd * ds * sp_softplus_grad(gam);
    }
  }
  __syncthreads();
  // 3. CTA partials of dlambda and dgamma (fixed order), dmetric out
  if (threadIdx.x == 0) {
    float s = 0.0f;
    for (int q = 0; q < np * N; ++q) s += sTl[q];
    dlam_part[cta] = s * (1.0f - tl * tl);
  }
  for (int n = threadIdx.x; n < N; n += SP_THREADS) {
    float s = 0.0f;
    for (int pl = 0; pl < np; ++pl) s += sGam[pl * N + n];
    dgam_part[cta * N + n] = s;
  }
  for (int t = threadIdx.x; t < N * T::TP; t += SP_THREADS) {
    const int n = t / T::TP, pl = t % T::TP;
    if (pl < np) dmraw[(b * N + n) * HW + p0 + pl] = sDm[n * T::LD + pl];
  }
  // 4. dC_in = dC + 0.5 tl (dpre - dpre^T), transposed into the C tile (read last in step 2)
  for (SpIter it(per_px); it.pl < np;) {
    int pls[SP_BATCH], rs[SP_BATCH];
    float dv[SP_BATCH];
#pragma unroll
    for (int u = 0; u < SP_BATCH; ++u) {
      pls[u] = it.pl;
      rs[u] = it.r;
      dv[u] = it.pl < np ? __ldg(d_c + base + it.pl * per_px + it.r) : 0.0f;
      it.next();
    }
#pragma unroll
    for (int u = 0; u < SP_BATCH; ++u) {
      const int pl = pls[u], r = rs[u];
      if (pl >= np) break;
      const int n = r / T::DD, ij = r % T::DD, i = ij / D, j = ij % D;
      const float h = 0.5f * sDs[n * T::LD + pl];
      const float dij = sG[pl * LG + r] * h, dji = sG[pl * LG + n * T::DD + j * D + i] * h;
      sC[r * T::LD + pl] = dv[u] + 0.5f * tl * (dij - dji);
    }
  }
  __syncthreads();
  // 5. NCHW gradients of the injection and generator convolutions (coalesced along pixels)
  for (int t = threadIdx.x; t < per_px * T::TP; t += SP_THREADS) {
    const int r = t / T::TP, pl = t % T::TP;
    if (pl < np) dcraw[(b * per_px + r) * HW + p0 + pl] = sC[r * T::LD + pl];
  }
  for (int t = threadIdx.x; t < N * T::K * T::TP; t += SP_THREADS) {
    const int r = t / T::TP, pl = t % T::TP;
    if (pl >= np) continue;
    const int n = r / T::K, k = r % T::K;
    const int u = sPair[0][k], v = sPair[1][k];
    const float h = 0.5f * sDs[n * T::LD + pl];
    const float* g = sG + pl * LG + n * T::DD;
    dbraw[(b * N * T::K + r) * HW + p0 + pl] = (g[u * D + v] - g[v * D + u]) * h;
  }
}

}  // namespace
}  // namespace csn

namespace {

using namespace csn;

constexpr size_t SP_SMEM_MAX = 227 * 1024 - 256;  // the backward also holds a static pair table

size_t sp_fwd_smem(int64_t N, int D) {
  const int64_t DD = D * D, K = D * (D - 1) / 2, TP = sp_tp(D);
  return (size_t)((N * DD + N * K + N) * (TP + 1)) * sizeof(float);
}

size_t sp_bwd_smem(int64_t N, int D) {
  const int64_t DD = D * D, K = D * (D - 1) / 2, TP = sp_tp(D);
  return (size_t)((N * DD + N * K + 3 * N) * (TP + 1) + TP * (N * DD + 1) + 2 * TP * N) * sizeof(float);
}

int sp_check(const char* fn, int64_t B, int64_t HW, int64_t N, int D) {
  char msg[192];
  if (D != 4 && D != 8 && D != 16) {
    snprintf(msg, sizeof msg, "%s: D = %d, expected 4, 8 or 16", fn, D);
    return set_error(CSN_ERR_UNSUPPORTED, msg);
  }
  // grid.x = ceil(HW / TP) with TP >= 16 must stay below 2^31: H*W <= 2^34
  if (B < 0 || HW < 0 || N < 0 || B > 65535 || HW > ((int64_t)1 << 34)) {
    snprintf(msg, sizeof msg, "%s: B in [0, 65535], H*W in [0, 2^34], N >= 0 required", fn);
    return set_error(CSN_ERR_INVALID, msg);
  }
  if (sp_bwd_smem(N, D) > SP_SMEM_MAX) {
    snprintf(msg, sizeof msg, "%s: N = %lld neurons of D = %d exceed one CTA's shared memory", fn, (long long)N, D);
    return set_error(CSN_ERR_UNSUPPORTED, msg);
  }
  return CSN_OK;
}

template <typename Kern>
int sp_smem_attr(Kern k, size_t bytes, const char* fn) {
  if (bytes <= 48 * 1024) return CSN_OK;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  return e == cudaSuccess ? CSN_OK : set_cuda_error(e, fn);
}

template <int D>
int sp_fwd(const float* craw, const float* braw, const float* mraw, const float* lam, const float* gam, float* om,
           float* c, float* dec, int64_t B, int64_t HW, int N, cudaStream_t st) {
  const size_t smem = sp_fwd_smem(N, D);
  if (int rc = sp_smem_attr(spatial_gen_fwd_kernel<D>, smem, "csn_spatial_generators_fwd")) return rc;
  const dim3 grid((unsigned)((HW + sp_tp(D) - 1) / sp_tp(D)), (unsigned)B);
  KernelTimer kt("spatial_generators_fwd", st);
  spatial_gen_fwd_kernel<D><<<grid, SP_THREADS, smem, st>>>(craw, braw, mraw, lam, gam, om, c, dec, HW, N);
  return check_launch("csn_spatial_generators_fwd");
}

template <int D>
int sp_bwd(const float* craw, const float* braw, const float* mraw, const float* lam, const float* gam,
           const float* dom, const float* dc, const float* ddec, float* dcraw, float* dbraw, float* dmraw,
           float* dlam, float* dgam, int64_t B, int64_t HW, int N, cudaStream_t st) {
  const size_t smem = sp_bwd_smem(N, D);
  if (int rc = sp_smem_attr(spatial_gen_bwd_kernel<D>, smem, "csn_spatial_generators_bwd")) return rc;
  const dim3 grid((unsigned)((HW + sp_tp(D) - 1) / sp_tp(D)), (unsigned)B);
  KernelTimer kt("spatial_generators_bwd", st);
  spatial_gen_bwd_kernel<D><<<grid, SP_THREADS, smem, st>>>(craw, braw, mraw, lam, gam, dom, dc, ddec, dcraw,
                                                             dbraw, dmraw, dlam, dgam, HW, N);
  return check_launch("csn_spatial_generators_bwd");
}

}  // namespace

extern "C" int64_t csn_spatial_generators_partials(int64_t B, int64_t HW, int D) {
  if (B < 0 || HW < 0 || (D != 4 && D != 8 && D != 16)) return 0;
  return B * ((HW + sp_tp(D) - 1) / sp_tp(D));
}

extern "C" int csn_spatial_generators_fwd(const float* in_proj, const float* biv_proj, const float* metric,
                                          const float* lambda_sw, const float* gamma_log, float* omega, float* c,
                                          float* decay, int64_t B, int64_t HW, int64_t N, int D, void* stream) {
  if (int rc = sp_check("csn_spatial_generators_fwd", B, HW, N, D)) return rc;
  if (B * HW * N == 0) return CSN_OK;
  if (!in_proj || !biv_proj || !metric || !lambda_sw || !gamma_log || !omega || !c || !decay)
    return set_error(CSN_ERR_INVALID, "csn_spatial_generators_fwd: missing pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int n = (int)N;
  if (D == 4) return sp_fwd<4>(in_proj, biv_proj, metric, lambda_sw, gamma_log, omega, c, decay, B, HW, n, st);
  if (D == 8) return sp_fwd<8>(in_proj, biv_proj, metric, lambda_sw, gamma_log, omega, c, decay, B, HW, n, st);
  return sp_fwd<16>(in_proj, biv_proj, metric, lambda_sw, gamma_log, omega, c, decay, B, HW, n, st);
}

extern "C" int csn_spatial_generators_bwd(const float* in_proj, const float* biv_proj, const float* metric,
                                          const float* lambda_sw, const float* gamma_log, const float* d_omega,
                                          const float* d_c, const float* d_decay, float* d_in_proj,
                                          float* d_biv_proj, float* d_metric, float* dlambda_part,
                                          float* dgamma_part, int64_t B, int64_t HW, int64_t N, int D,
                                          void* stream) {
  if (int rc = sp_check("csn_spatial_generators_bwd", B, HW, N, D)) return rc;
  if (B * HW * N == 0) {
    // no neurons: the lambda partials (one per CTA tile) are still summed by the caller
    const int64_t P = csn_spatial_generators_partials(B, HW, D);
    if (P > 0 && dlambda_part) {
      cudaError_t e = cudaMemsetAsync(dlambda_part, 0, sizeof(float) * P, static_cast<cudaStream_t>(stream));
      if (e != cudaSuccess) return set_cuda_error(e, "csn_spatial_generators_bwd: cudaMemsetAsync");
    }
    return CSN_OK;
  }
  if (!in_proj || !biv_proj || !metric || !lambda_sw || !gamma_log || !d_omega || !d_c || !d_decay || !d_in_proj ||
      !d_biv_proj || !d_metric || !dlambda_part || !dgamma_part)
    return set_error(CSN_ERR_INVALID, "csn_spatial_generators_bwd: missing pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int n = (int)N;
  if (D == 4)
    return sp_bwd<4>(in_proj, biv_proj, metric, lambda_sw, gamma_log, d_omega, d_c, d_decay, d_in_proj, d_biv_proj,
                     d_metric, dlambda_part, dgamma_part, B, HW, n, st);
  if (D == 8)
    return sp_bwd<8>(in_proj, biv_proj, metric, lambda_sw, gamma_log, d_omega, d_c, d_decay, d_in_proj, d_biv_proj,
                     d_metric, dlambda_part, dgamma_part, B, HW, n, st);
  return sp_bwd<16>(in_proj, biv_proj, metric, lambda_sw, gamma_log, d_omega, d_c, d_decay, d_in_proj, d_biv_proj,
                    d_metric, dlambda_part, dgamma_part, B, HW, n, st);
}
