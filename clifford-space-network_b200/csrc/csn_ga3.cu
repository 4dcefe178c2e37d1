// csn_ga3.cu -- Cl(3,0) affine rotor scan in the blade basis.
//
//   h_t = R_t h_{t-1} R~_t + x_t,   h_{-1} = h0 (or 0)
//   R_t = (1 - Om)^{-1} (1 + Om) = (1 - |Om|^2 + 2 Om) / (1 + |Om|^2),  Om = dt/2 (g12 e12 + g23 e23 + g31 e31)
// Multivectors use the layout [1, e1, e2, e3, e12, e23, e31, e123]
// (include/clifford_configs.cuh:38-51); rotors are even elements [1, e12, e23, e31].
// The sandwich v -> R v R~ is the 8 x 8 linear map generated in ga_tables.h from the
// blade product table (block diagonal by grade, 20 nonzeros).  A unit rotor makes it
// orthogonal, so its transpose R~ v R is the adjoint map used by the backward pass.
//
// Same reduce -> carry -> apply chunking as the matrix scans; the scan element is
// (rotor P: 4 floats, offset c: 8 floats) and composes as (P2 P1, P2 c1 P2~ + c2).
#include "csn_common.cuh"
#include "csn_internal.h"

namespace csn {
namespace ga3 {

struct Args {
  const float* gens;  // [B, T, N, 3]
  const float* dt;    // [B, T]
  const float* x;     // [B, T, N, 8]
  const float* h0;    // [B, N, 8] or null
  const float* h;     // forward output (backward)
  const float* dh;    // [B, T, N, 8] (backward)
  float* out;         // forward h
  float* dx;          // backward
  float* dgens;
  float* ddt_part;    // [B, T, N]
  float* ddt;         // [B, T]
  float* dh0;
  float* aggP;   // [S, nchunks, 4]
  float* aggC;   // [S, nchunks, 8]
  float* carry;  // [S, nchunks, 8]
  int64_t B, T, N, nchunks, chunk;
};

__device__ __forceinline__ void load8(float (&v)[8], const float* __restrict__ p) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void store8(float* __restrict__ p, const float (&v)[8]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}
__device__ __forceinline__ void store8_cs(float* __restrict__ p, const float (&v)[8]) {
  __stcs(reinterpret_cast<float4*>(p), make_float4(v[0], v[1], v[2], v[3]));
  __stcs(reinterpret_cast<float4*>(p) + 1, make_float4(v[4], v[5], v[6], v[7]));
}

// Rotor of step (g, dt) from the generator values; also returns Om and w = |Om|^2 for the
// backward pass.
__device__ __forceinline__ void rotor_vals(const float (&g)[3], float dtv, float (&r)[4], float (&om)[3],
                                           float& w) {
  const float hh = 0.5f * dtv;
  om[0] = hh * g[0];
  om[1] = hh * g[1];
  om[2] = hh * g[2];
  w = om[0] * om[0] + om[1] * om[1] + om[2] * om[2];
  const float inv = 1.0f / (1.0f + w);
  r[0] = 1.0f - 2.0f * w * inv;  // (1 - w) / (1 + w), rounded once near 1
  r[1] = 2.0f * om[0] * inv;
  r[2] = 2.0f * om[1] * inv;
  r[3] = 2.0f * om[2] * inv;
}
// the same from the generators in memory
__device__ __forceinline__ void rotor(const float* __restrict__ g, float dtv, float (&r)[4],
                                      float (&om)[3], float& w) {
  const float gv[3] = {__ldg(g), __ldg(g + 1), __ldg(g + 2)};
  rotor_vals(gv, dtv, r, om, w);
}

// y = L x   and   y = L^T x   for the sandwich map L
__device__ __forceinline__ void apply_L(const Ga3Map& L, const float (&v)[8], float (&y)[8]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) s = fmaf(L.m[i][j], v[j], s);  // zeros fold away
    y[i] = s;
  }
}
__device__ __forceinline__ void apply_LT(const Ga3Map& L, const float (&v)[8], float (&y)[8]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) s = fmaf(L.m[i][j], v[i], s);
    y[j] = s;
  }
}

__device__ __forceinline__ void coords(const Args& a, int64_t tid, int64_t& b, int64_t& n, int64_t& j) {
  n = tid % a.N;
  j = (tid / a.N) % a.nchunks;
  b = tid / (a.N * a.nchunks);
}

// forward chunk aggregate: P = R_end ... R_start (even product), c = local scan
__global__ void __launch_bounds__(256) fwd_reduce(Args a) {
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (tid >= a.B * a.N * a.nchunks) return;
  int64_t b, n, j;
  coords(a, tid, b, n, j);
  const int64_t t0 = j * a.chunk, t1 = min(a.T, t0 + a.chunk);
  float P[4] = {1.0f, 0.0f, 0.0f, 0.0f}, c[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  // the next step's inputs are loaded while this step is computed (the pass reads 44 bytes per
  // step and does little arithmetic on them: without the overlap it waits on every load)
  float gn[3], dn = 0.0f, xn[8];
  auto fetch = [&](int64_t t) {
    const int64_t e = (b * a.T + t) * a.N + n;
    gn[0] = __ldg(a.gens + e * 3); gn[1] = __ldg(a.gens + e * 3 + 1); gn[2] = __ldg(a.gens + e * 3 + 2);
    dn = __ldg(a.dt + b * a.T + t);
    load8(xn, a.x + e * 8);
  };
  if (t0 < t1) fetch(t0);
  for (int64_t t = t0; t < t1; ++t) {
    float g[3] = {gn[0], gn[1], gn[2]}, xv[8];
    const float dtv = dn;
#pragma unroll
    for (int i = 0; i < 8; ++i) xv[i] = xn[i];
    if (t + 1 < t1) fetch(t + 1);
    float r[4], om[3], w, y[8];
    rotor_vals(g, dtv, r, om, w);
    Ga3Map L;
    ga3_sandwich_matrix(r[0], r[1], r[2], r[3], L);
    apply_L(L, c, y);
#pragma unroll
    for (int i = 0; i < 8; ++i) c[i] = y[i] + xv[i];
    float Pn[4];
    ga3_even_mul(r, P, Pn);
#pragma unroll
    for (int i = 0; i < 4; ++i) P[i] = Pn[i];
  }
  const int64_t s = b * a.N + n;
  reinterpret_cast<float4*>(a.aggP)[s * a.nchunks + j] = make_float4(P[0], P[1], P[2], P[3]);
  store8(a.aggC + (s * a.nchunks + j) * 8, c);
}

// ------------------------------------------------------- carries, warp per sequence
// The carry is a chain of links over the chunks of a sequence: forward h <- L(P_j) h + c_j
// (j = 0 .. nchunks-2, from h0), backward H <- L(P_j)^T H + c'_j (j = nchunks-1 .. 1, from
// zero).  A warp walks it in three phases instead of one thread walking every link:
//   1. lane l composes its contiguous range of ~(nchunks-1)/32 links into one link
//   2. an inclusive shuffle scan over the 32 lanes (5 levels) composes each lane's link
//      after those of the lanes before it
//   3. lane l takes its carry-in from lane l-1's prefix and replays its range, writing
//      every carry
// Forward composition, A then B: (P_B P_A, L(P_B) c_A + c_B).  Backward, with the map
// H -> L(Q)^T H + c: A then B gives (Q_A Q_B, L(Q_B)^T c_A + c_B).  Each lane's aggregates
// are read through a ring of CARRY_PF links in flight.
constexpr int CARRY_PF = 4;

template <bool REV>
__device__ __forceinline__ void link_apply(const float (&q)[4], const float (&v)[8], float (&y)[8]) {
  Ga3Map L;
  ga3_sandwich_matrix(q[0], q[1], q[2], q[3], L);
  if constexpr (REV) apply_LT(L, v, y);
  else apply_L(L, v, y);
}

// (q, c) <- (q, c) after (p, cp): forward (q p, L(q) cp + c), backward (p q, L(q)^T cp + c)
template <bool REV>
__device__ __forceinline__ void compose_after(float (&q)[4], float (&c)[8], const float (&p)[4],
                                              const float (&cp)[8]) {
  float y[8], qn[4];
  link_apply<REV>(q, cp, y);
#pragma unroll
  for (int i = 0; i < 8; ++i) c[i] += y[i];
  if constexpr (REV) ga3_even_mul(p, q, qn);
  else ga3_even_mul(q, p, qn);
#pragma unroll
  for (int i = 0; i < 4; ++i) q[i] = qn[i];
}

template <bool REV>
__global__ void __launch_bounds__(128) carry_warp(Args a) {
  const int64_t s = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (s >= a.B * a.N) return;  // s is the same for the whole warp
  const int64_t nch = a.nchunks, nl = nch - 1;
  const int64_t per = (nl + 31) / 32;
  const int64_t k0 = min(nl, lane * per), k1 = min(nl, k0 + per);
  const float4* aggP = reinterpret_cast<const float4*>(a.aggP) + s * nch;
  const float* aggC = a.aggC + s * nch * 8;
  float* carry = a.carry + s * nch * 8;
  // link k: forward chunk k -> carry k + 1; backward chunk nch-1-k -> carry nch-2-k
  auto chunk_of = [&](int64_t k) { return REV ? nch - 1 - k : k; };
  auto out_of = [&](int64_t k) { return REV ? nch - 2 - k : k + 1; };
  float rp[CARRY_PF][4], rc[CARRY_PF][8];
  auto fetch = [&](int64_t k, int u) {
    const float4 q = aggP[chunk_of(k)];
    rp[u][0] = q.x; rp[u][1] = q.y; rp[u][2] = q.z; rp[u][3] = q.w;
    load8(rc[u], aggC + chunk_of(k) * 8);
  };
  auto prefetch = [&]() {
#pragma unroll
    for (int u = 0; u < CARRY_PF; ++u)
      if (k0 + u < k1) fetch(k0 + u, u);
  };
  // 1. the lane's range as one link, from the identity
  float q[4] = {1.0f, 0.0f, 0.0f, 0.0f}, c[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  prefetch();
  for (int64_t kk = k0; kk < k1; kk += CARRY_PF) {
#pragma unroll
    for (int u = 0; u < CARRY_PF; ++u) {
      const int64_t k = kk + u;
      if (k >= k1) break;
      float p[4], cp[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) p[i] = rp[u][i];
#pragma unroll
      for (int i = 0; i < 8; ++i) cp[i] = rc[u][i];
      if (k + CARRY_PF < k1) fetch(k + CARRY_PF, u);
      // this link after the range so far: (p, c_k) after (q, c)
      float y[8], qn[4];
      link_apply<REV>(p, c, y);
#pragma unroll
      for (int i = 0; i < 8; ++i) c[i] = y[i] + cp[i];
      if constexpr (REV) ga3_even_mul(q, p, qn);
      else ga3_even_mul(p, q, qn);
#pragma unroll
      for (int i = 0; i < 4; ++i) q[i] = qn[i];
    }
  }
  prefetch();  // the replay's first links are in flight during the scan
  // 2. inclusive scan over the lanes
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    float pp[4], cp[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) pp[i] = __shfl_up_sync(0xffffffffu, q[i], d);
#pragma unroll
    for (int i = 0; i < 8; ++i) cp[i] = __shfl_up_sync(0xffffffffu, c[i], d);
    if (lane >= d) compose_after<REV>(q, c, pp, cp);
  }
  // 3. carry-in: the initial state through the links of lanes 0 .. l-1
  float pe[4], ce[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) pe[i] = __shfl_up_sync(0xffffffffu, q[i], 1);
#pragma unroll
  for (int i = 0; i < 8; ++i) ce[i] = __shfl_up_sync(0xffffffffu, c[i], 1);
  float h[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  const float* init = REV ? nullptr : a.h0;
  if (init) load8(h, init + s * 8);
  if (lane == 0) store8(carry + (REV ? nch - 1 : 0) * 8, h);
  if (lane > 0) {
    float y[8];
    if (init) link_apply<REV>(pe, h, y);
    else {
#pragma unroll
      for (int i = 0; i < 8; ++i) y[i] = 0.0f;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) h[i] = y[i] + ce[i];
  }
  for (int64_t kk = k0; kk < k1; kk += CARRY_PF) {
#pragma unroll
    for (int u = 0; u < CARRY_PF; ++u) {
      const int64_t k = kk + u;
      if (k >= k1) break;
      float p[4], cp[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) p[i] = rp[u][i];
#pragma unroll
      for (int i = 0; i < 8; ++i) cp[i] = rc[u][i];
      if (k + CARRY_PF < k1) fetch(k + CARRY_PF, u);
      float y[8];
      link_apply<REV>(p, h, y);
#pragma unroll
      for (int i = 0; i < 8; ++i) h[i] = y[i] + cp[i];
      store8(carry + out_of(k) * 8, h);
    }
  }
}

__global__ void __launch_bounds__(256) fwd_apply(Args a) {
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (tid >= a.B * a.N * a.nchunks) return;
  int64_t b, n, j;
  coords(a, tid, b, n, j);
  const int64_t s = b * a.N + n;
  const int64_t t0 = j * a.chunk, t1 = min(a.T, t0 + a.chunk);
  float h[8];
  if (a.nchunks > 1) load8(h, a.carry + (s * a.nchunks + j) * 8);
  else if (a.h0) load8(h, a.h0 + s * 8);
  else {
#pragma unroll
    for (int i = 0; i < 8; ++i) h[i] = 0.0f;
  }
  for (int64_t t = t0; t < t1; ++t) {
    const int64_t e = (b * a.T + t) * a.N + n;
    float r[4], om[3], w, y[8], xv[8];
    rotor(a.gens + e * 3, __ldg(a.dt + b * a.T + t), r, om, w);
    Ga3Map L;
    ga3_sandwich_matrix(r[0], r[1], r[2], r[3], L);
    apply_L(L, h, y);
    load8(xv, a.x + e * 8);
#pragma unroll
    for (int i = 0; i < 8; ++i) h[i] = y[i] + xv[i];
    store8_cs(a.out + e * 8, h);
  }
}

// backward chunk aggregate: g <- 0; for t = end..start: G = dh_t + g; g = L_t^T G;  P as forward
__global__ void __launch_bounds__(256) bwd_reduce(Args a) {
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (tid >= a.B * a.N * a.nchunks) return;
  int64_t b, n, j;
  coords(a, tid, b, n, j);
  if (j == 0) return;
  const int64_t t0 = j * a.chunk, t1 = min(a.T, t0 + a.chunk);
  float P[4] = {1.0f, 0.0f, 0.0f, 0.0f}, g[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  float gn[3], dn = 0.0f, vn[8];  // next step's inputs, loaded a step ahead
  auto fetch = [&](int64_t t) {
    const int64_t e = (b * a.T + t) * a.N + n;
    gn[0] = __ldg(a.gens + e * 3); gn[1] = __ldg(a.gens + e * 3 + 1); gn[2] = __ldg(a.gens + e * 3 + 2);
    dn = __ldg(a.dt + b * a.T + t);
    load8(vn, a.dh + e * 8);
  };
  if (t0 < t1) fetch(t1 - 1);
  for (int64_t t = t1 - 1; t >= t0; --t) {
    float gg[3] = {gn[0], gn[1], gn[2]}, dv[8];
    const float dtv = dn;
#pragma unroll
    for (int i = 0; i < 8; ++i) dv[i] = vn[i];
    if (t - 1 >= t0) fetch(t - 1);
    float r[4], om[3], w, y[8];
    rotor_vals(gg, dtv, r, om, w);
    Ga3Map L;
    ga3_sandwich_matrix(r[0], r[1], r[2], r[3], L);
#pragma unroll
    for (int i = 0; i < 8; ++i) dv[i] += g[i];
    apply_LT(L, dv, y);
#pragma unroll
    for (int i = 0; i < 8; ++i) g[i] = y[i];
    float Pn[4];
    ga3_even_mul(P, r, Pn);  // P <- P R (reverse accumulation of R_end ... R_start)
#pragma unroll
    for (int i = 0; i < 4; ++i) P[i] = Pn[i];
  }
  const int64_t s = b * a.N + n;
  reinterpret_cast<float4*>(a.aggP)[s * a.nchunks + j] = make_float4(P[0], P[1], P[2], P[3]);
  store8(a.aggC + (s * a.nchunks + j) * 8, g);
}

__global__ void __launch_bounds__(256) bwd_apply(Args a) {
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (tid >= a.B * a.N * a.nchunks) return;
  int64_t b, n, j;
  coords(a, tid, b, n, j);
  const int64_t s = b * a.N + n;
  const int64_t t0 = j * a.chunk, t1 = min(a.T, t0 + a.chunk);
  float H[8];
  if (a.nchunks > 1) load8(H, a.carry + (s * a.nchunks + j) * 8);
  else {
#pragma unroll
    for (int i = 0; i < 8; ++i) H[i] = 0.0f;
  }
  for (int64_t t = t1 - 1; t >= t0; --t) {
    const int64_t e = (b * a.T + t) * a.N + n;
    const float dtv = __ldg(a.dt + b * a.T + t);
    float r[4], om[3], w, G[8], hp[8], dr[4];
    rotor(a.gens + e * 3, dtv, r, om, w);
    load8(G, a.dh + e * 8);
#pragma unroll
    for (int i = 0; i < 8; ++i) G[i] += H[i];
    store8_cs(a.dx + e * 8, G);
    if (t > 0) load8(hp, a.h + ((b * a.T + t - 1) * a.N + n) * 8);
    else if (a.h0) load8(hp, a.h0 + s * 8);
    else {
#pragma unroll
      for (int i = 0; i < 8; ++i) hp[i] = 0.0f;
    }
    ga3_sandwich_vjp(r[0], r[1], r[2], r[3], hp, G, dr);
    // r0 = (1 - w)/(1 + w), r_b = 2 om_b / (1 + w)
    const float den = 1.0f / (1.0f + w), den2 = den * den;
    float dom[3];
#pragma unroll
    for (int bb = 0; bb < 3; ++bb) {
      float v = dr[0] * (-4.0f * om[bb] * den2);
#pragma unroll
      for (int c = 0; c < 3; ++c) v = fmaf(dr[1 + c], ((bb == c) ? 2.0f * den : 0.0f) - 4.0f * om[c] * om[bb] * den2, v);
      dom[bb] = v;
    }
    const float* gp = a.gens + e * 3;
    float* dg = a.dgens + e * 3;
    float ddt = 0.0f;
#pragma unroll
    for (int bb = 0; bb < 3; ++bb) {
      dg[bb] = 0.5f * dtv * dom[bb];
      ddt = fmaf(0.5f * __ldg(gp + bb), dom[bb], ddt);
    }
    a.ddt_part[e] = ddt;
    Ga3Map L;
    ga3_sandwich_matrix(r[0], r[1], r[2], r[3], L);
    apply_LT(L, G, H);
  }
  if (j == 0 && a.dh0) store8(a.dh0 + s * 8, H);
}

__global__ void reduce_channels(const float* __restrict__ part, float* __restrict__ out, int64_t BT,
                                int64_t N) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= BT) return;
  const float* p = part + i * N;
  float s = 0.0f;
  if ((N & 3) == 0 && (reinterpret_cast<uintptr_t>(p) & 15u) == 0) {
    // the same left-to-right sum from 16-byte loads
    for (int64_t n = 0; n < N; n += 4) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(p + n));
      s += v.x;
      s += v.y;
      s += v.z;
      s += v.w;
    }
  } else {
    for (int64_t n = 0; n < N; ++n) s += p[n];
  }
  out[i] = s;
}

struct Plan {
  int64_t chunk, nchunks;
  size_t floats;  // aggP + aggC + carry (+ ddt partials)
};

Plan plan(int64_t B, int64_t T, int64_t N, bool bwd) {
  Plan p;
  const int64_t S = B * N;
  // two waves at 2048 threads per SM: the apply passes hold 768 - 1536 threads / SM
  // (40 - 77 registers), and halving the chunk shortens their last wave's tail (Cl(3)
  // B64 L65536 C16: 3.80 -> 3.71 ms per step; 4x as many chunks, 3.75)
  const int64_t target = 148 * 4096;
  p.chunk = (S * T + target - 1) / target;
  if (p.chunk < 16) p.chunk = 16;
  if (p.chunk > T) p.chunk = T > 0 ? T : 1;
  p.nchunks = T > 0 ? (T + p.chunk - 1) / p.chunk : 0;
  p.floats = (p.nchunks > 1 ? (size_t)S * p.nchunks * 20 : 0) + (bwd ? (size_t)B * T * N : 0);
  return p;
}

size_t plan_bytes(const Plan& p) { return p.floats * sizeof(float) + 512; }

void bind(Args& a, const Plan& p, float* base) {
  const int64_t S = a.B * a.N;
  float* al = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(base) + 255) & ~uintptr_t(255));
  const size_t one = p.nchunks > 1 ? (size_t)S * p.nchunks : 0;
  a.aggP = al;
  a.aggC = al + 4 * one;
  a.carry = al + 12 * one;
  a.ddt_part = al + 20 * one;
  a.chunk = p.chunk;
  a.nchunks = p.nchunks;
}

unsigned blocks(int64_t n, int t) { return (unsigned)((n + t - 1) / t); }

}  // namespace ga3
}  // namespace csn

using namespace csn;

extern "C" size_t csn_ga3_workspace_bytes(int64_t B, int64_t T, int64_t N) {
  if (B < 0 || T < 0 || N < 0) return 0;
  return ga3::plan_bytes(ga3::plan(B, T, N, true));
}

static int ga3_ws(void* user, size_t bytes, size_t need, cudaStream_t st, float** out, bool* owned) {
  *owned = false;
  if (user) {
    if (bytes < need) return set_error(CSN_ERR_INVALID, "Cl(3) scan: workspace too small");
    *out = static_cast<float*>(user);
    return CSN_OK;
  }
  cudaError_t e = cudaMallocAsync(reinterpret_cast<void**>(out), need, st);
  if (e != cudaSuccess) return set_cuda_error(e, "Cl(3) scan: cudaMallocAsync");
  *owned = true;
  return CSN_OK;
}

static bool ga3_al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

extern "C" int csn_ga3_scan_fwd(const float* gens, const float* dt, const float* x, const float* h0,
                                float* h, int64_t B, int64_t T, int64_t N, void* workspace,
                                size_t workspace_bytes, void* stream) {
  if (B < 0 || T < 0 || N < 0) return set_error(CSN_ERR_INVALID, "csn_ga3_scan_fwd: negative size");
  if (B * T * N == 0) return CSN_OK;
  if (!gens || !dt || !x || !h) return set_error(CSN_ERR_INVALID, "csn_ga3_scan_fwd: missing pointer");
  if (!ga3_al16(x) || !ga3_al16(h) || (h0 && !ga3_al16(h0)))
    return set_error(CSN_ERR_INVALID, "csn_ga3_scan_fwd: x, h, h0 must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  ga3::Plan p = ga3::plan(B, T, N, false);
  float* ws;
  bool owned;
  if (int rc = ga3_ws(workspace, workspace_bytes, ga3::plan_bytes(p), st, &ws, &owned)) return rc;
  ga3::Args a{};
  a.gens = gens; a.dt = dt; a.x = x; a.h0 = h0; a.out = h; a.B = B; a.T = T; a.N = N;
  ga3::bind(a, p, ws);
  const int64_t S = B * N, total = S * p.nchunks;
  if (p.nchunks > 1) {
    {
      KernelTimer kt("ga3_fwd_reduce", st);
      ga3::fwd_reduce<<<ga3::blocks(total, 256), 256, 0, st>>>(a);
    }
    KernelTimer kt("ga3_fwd_carry", st);
    ga3::carry_warp<false><<<ga3::blocks(S * 32, 128), 128, 0, st>>>(a);
  }
  {
    KernelTimer kt("ga3_fwd_apply", st);
    ga3::fwd_apply<<<ga3::blocks(total, 256), 256, 0, st>>>(a);
  }
  int rc = check_launch("csn_ga3_scan_fwd");
  if (owned) cudaFreeAsync(ws, st);
  return rc;
}

extern "C" int csn_ga3_scan_bwd(const float* gens, const float* dt, const float* h0, const float* h,
                                const float* dh, float* dgens, float* ddt, float* dx, float* dh0,
                                int64_t B, int64_t T, int64_t N, void* workspace,
                                size_t workspace_bytes, void* stream) {
  if (B < 0 || T < 0 || N < 0) return set_error(CSN_ERR_INVALID, "csn_ga3_scan_bwd: negative size");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (B * T * N == 0) {
    if (B * T > 0 && ddt) {
      cudaError_t e = cudaMemsetAsync(ddt, 0, sizeof(float) * B * T, st);
      if (e != cudaSuccess) return set_cuda_error(e, "csn_ga3_scan_bwd: cudaMemsetAsync");
    }
    return CSN_OK;
  }
  if (!gens || !dt || !h || !dh || !dgens || !ddt || !dx)
    return set_error(CSN_ERR_INVALID, "csn_ga3_scan_bwd: missing pointer");
  if (dh0 && !h0) return set_error(CSN_ERR_INVALID, "csn_ga3_scan_bwd: dh0 needs h0");
  if (!ga3_al16(h) || !ga3_al16(dh) || !ga3_al16(dx) || (h0 && !ga3_al16(h0)) || (dh0 && !ga3_al16(dh0)))
    return set_error(CSN_ERR_INVALID, "csn_ga3_scan_bwd: 16-byte alignment required");
  ga3::Plan p = ga3::plan(B, T, N, true);
  float* ws;
  bool owned;
  if (int rc = ga3_ws(workspace, workspace_bytes, ga3::plan_bytes(p), st, &ws, &owned)) return rc;
  ga3::Args a{};
  a.gens = gens; a.dt = dt; a.h0 = h0; a.h = h; a.dh = dh; a.dgens = dgens; a.ddt = ddt; a.dx = dx;
  a.dh0 = dh0; a.B = B; a.T = T; a.N = N;
  ga3::bind(a, p, ws);
  const int64_t S = B * N, total = S * p.nchunks;
  if (p.nchunks > 1) {
    {
      KernelTimer kt("ga3_bwd_reduce", st);
      ga3::bwd_reduce<<<ga3::blocks(total, 256), 256, 0, st>>>(a);
    }
    KernelTimer kt("ga3_bwd_carry", st);
    ga3::carry_warp<true><<<ga3::blocks(S * 32, 128), 128, 0, st>>>(a);
  }
  {
    KernelTimer kt("ga3_bwd_apply", st);
    ga3::bwd_apply<<<ga3::blocks(total, 256), 256, 0, st>>>(a);
  }
  {
    KernelTimer kt("ga3_reduce_channels", st);
    ga3::reduce_channels<<<ga3::blocks(B * T, 256), 256, 0, st>>>(a.ddt_part, ddt, B * T, N);
  }
  int rc = check_launch("csn_ga3_scan_bwd");
  if (owned) cudaFreeAsync(ws, st);
  return rc;
}
