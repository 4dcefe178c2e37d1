// csn_scan16.cu -- D = 16 (Cl(8,0) ~ M_16(R)) scans on warp-level tensor-core MMA.
//
// Same chunked reduce -> carry -> apply algorithm as the other families, one warp per
// (sequence, chunk).  A 16 x 16 matrix lives in registers as an mma.m16n8k8 accumulator
// fragment ("F16", 8 floats per lane): lane (g = lane / 4, t = lane % 4) holds rows g and
// g + 8 at columns 8 nt + 2 t and 8 nt + 2 t + 1 of each 8-column half nt.  Those same
// registers are the row-major A operand of mma.m16n8k8.tf32 when the k index inside each
// k-step is permuted as (slot t, slot t + 4) <-> (column 2 t, column 2 t + 1), and the
// B operand of the TRANSPOSED matrix under the same permutation.  So a product of the
// form Z = A B^T takes two fragments and yields a fragment with no data movement, and
// every product of the scan is written that way:
//   forward      X' = M (M X^T)^T + C            (two products)
//   chunk product P^T <- P^T M^T
//   adjoint      H' = M^T (M^T G^T)^T,  dM = (G M) Xp^T + G^T (Xp^T M^T)^T, ...
// Two tensor-core precisions, chosen by where a product's rounding error goes:
//  * the recurrent products -- the state X, the chunk product P, the gradient carry H
//    and g -- feed the next step, so their rounding errors accumulate over the whole
//    sequence.  The tf32 MMA's fp32 accumulation truncates toward zero (about -0.3 ulp
//    per MMA, -1 ulp with a chained C, measured on sm_100a), which shrinks an undamped
//    state by a few ulps per step: 5e-4 off the float64 recurrence after 8192 steps at
//    the Cl(8,0) benchmark shape.  These products therefore run on the FP64 tensor
//    cores (mma.m8n8k4.f64 on f64 copies of the same fragments, "F16D"): exact fp32
//    inputs, fp64 accumulation, one round-to-nearest when a value goes back to fp32;
//  * the per-step adjoint products (dM, dOmega) do not feed the recurrence and run as
//    3xTF32: each fp32 operand is split into a TF32 head and a TF32 tail and
//    hi*hi + hi*lo + lo*hi is accumulated in fp32 (fp32-level error, no accumulation over
//    time).  Transposes are data movement (two shuffle rounds per 8 x 8 tile), not
//    products: exact, and off the tensor pipes.
// The Cayley rotor is built from E = (I - Omega)^{-1} - I: a matrix series of small
// products when |h Omega|_F <= 0.05, else a Gauss-Jordan elimination on the fragment in
// deviation form (round-to-nearest FMAs), whose pivot rows and columns reach the lanes that
// need them by shuffles; the step stays in registers.
#include <stdint.h>

#include "csn_common.cuh"
#include "csn_internal.h"
#include "csn_scan_args.cuh"
#include "csn_carry.cuh"

namespace csn {
namespace s16 {

constexpr int D = 16;
constexpr int DD = 256;
constexpr int WARPS = 4;   // warps per block
constexpr int ZST = 20;    // row stride of the dOmega scratch (20 = 8t + g spreads banks)
constexpr unsigned FULL = 0xffffffffu;

// ------------------------------------------------------------------- fragments
struct F16 {
  float v[2][4];  // v[nt][e]: row g + 8 (e >> 1), column 8 nt + 2 t + (e & 1)
};
struct F16S {      // 3xTF32 operand: head and tail of every element
  uint32_t hi[2][4], lo[2][4];
};

__device__ __forceinline__ int frow(int lane, int e) { return (lane >> 2) + 8 * (e >> 1); }
__device__ __forceinline__ int fcol(int lane, int nt, int e) { return 8 * nt + 2 * (lane & 3) + (e & 1); }

// Head = x rounded to TF32 (nearest, ties away from zero: add half a TF32 unit to the
// magnitude bits and clear the 13 bits below the TF32 mantissa); tail = x - head, which
// is exact in fp32 and is read by the MMA at TF32 precision.
__device__ __forceinline__ void split(F16S& o, const F16& x) {
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint32_t h = (__float_as_uint(x.v[nt][e]) + 0x1000u) & 0xffffe000u;
      o.hi[nt][e] = h;
      o.lo[nt][e] = __float_as_uint(x.v[nt][e] - __uint_as_float(h));
    }
}

// d (16 x 8) += A (16 x 8) * B (8 x 8), TF32 inputs, fp32 accumulation.
__device__ __forceinline__ void mma_tf32(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// z = A B^T (3xTF32).  A fragment of k-step ks: (v[ks][0], v[ks][2], v[ks][1], v[ks][3]);
// B fragment of (k-step ks, output half nz): (v[ks][2 nz], v[ks][2 nz + 1]).
__device__ __forceinline__ void nt(F16& z, const F16S& A, const F16S& B) {
#pragma unroll
  for (int nz = 0; nz < 2; ++nz) {
    float d0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, d1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) {
      const uint32_t bh0 = B.hi[ks][2 * nz], bh1 = B.hi[ks][2 * nz + 1];
      const uint32_t bl0 = B.lo[ks][2 * nz], bl1 = B.lo[ks][2 * nz + 1];
      mma_tf32(d0, A.hi[ks][0], A.hi[ks][2], A.hi[ks][1], A.hi[ks][3], bh0, bh1);
      mma_tf32(d1, A.hi[ks][0], A.hi[ks][2], A.hi[ks][1], A.hi[ks][3], bl0, bl1);
      mma_tf32(d1, A.lo[ks][0], A.lo[ks][2], A.lo[ks][1], A.lo[ks][3], bh0, bh1);
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) z.v[nz][e] = d0[e] + d1[e];
  }
}

// z = A B^T with one TF32 product per k-step: A's head times B as given (the MMA reads
// the TF32 part of each fp32 entry, the low 13 bits are ignored).  Only for products many
// binades below the fp32 rounding of the sum they enter.
__device__ __forceinline__ void nt_head(F16& z, const F16S& A, const F16& B) {
#pragma unroll
  for (int nz = 0; nz < 2; ++nz) {
    float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int ks = 0; ks < 2; ++ks)
      mma_tf32(d, A.hi[ks][0], A.hi[ks][2], A.hi[ks][1], A.hi[ks][3], __float_as_uint(B.v[ks][2 * nz]),
               __float_as_uint(B.v[ks][2 * nz + 1]));
#pragma unroll
    for (int e = 0; e < 4; ++e) z.v[nz][e] = d[e];
  }
}

// z = X^T by data movement.  Tile (I, J) of z is tile (J, I) of X transposed; an 8 x 8
// tile, of which lane (g, t) holds row g at columns 2t and 2t + 1, turns in two shuffle
// rounds: lanes g and g ^ 1 swap one entry each so that lane (g, t) holds column
// 2t + (g & 1) at rows g & ~1 and (g & ~1) + 1, and the lane that needs column g' at rows
// 2t', 2t' + 1 reads both from lane 4 (2t' + (g' & 1)) + g' / 2.
template <typename V>
__device__ __forceinline__ void transpose_tiles(V (&z)[2][4], const V (&x)[2][4], int lane) {
  const int g = lane >> 2, t = lane & 3;
  const bool odd = g & 1;
  const int src = 4 * (2 * t + (g & 1)) + (g >> 1);
#pragma unroll
  for (int I = 0; I < 2; ++I)
#pragma unroll
    for (int J = 0; J < 2; ++J) {
      const V a0 = x[I][2 * J], a1 = x[I][2 * J + 1];  // tile (J, I) of X
      const V r = __shfl_xor_sync(FULL, odd ? a0 : a1, 4);
      const V b0 = odd ? r : a0, b1 = odd ? a1 : r;
      z[J][2 * I] = __shfl_sync(FULL, b0, src);
      z[J][2 * I + 1] = __shfl_sync(FULL, b1, src);
    }
}
__device__ __forceinline__ void transpose(F16& z, const F16& x, int lane) { transpose_tiles(z.v, x.v, lane); }

__device__ __forceinline__ void f_zero(F16& x) {
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) x.v[nt][e] = 0.0f;
}
__device__ __forceinline__ void f_identity(F16& x, int lane) {
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) x.v[nt][e] = (frow(lane, e) == fcol(lane, nt, e)) ? 1.0f : 0.0f;
}
// row-major 16 x 16 at p (8-byte aligned)
__device__ __forceinline__ void f_load(F16& x, const float* __restrict__ p, int lane) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float2 v = __ldg(reinterpret_cast<const float2*>(p + (g + 8 * h) * 16 + 8 * nt + 2 * t));
      x.v[nt][2 * h] = v.x;
      x.v[nt][2 * h + 1] = v.y;
    }
}
__device__ __forceinline__ void f_load_plain(F16& x, const float* p, int lane) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float2 v = *reinterpret_cast<const float2*>(p + (g + 8 * h) * 16 + 8 * nt + 2 * t);
      x.v[nt][2 * h] = v.x;
      x.v[nt][2 * h + 1] = v.y;
    }
}
template <bool STREAM>
__device__ __forceinline__ void f_store(float* p, const F16& x, int lane, float scale = 1.0f) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float2 v = make_float2(scale * x.v[nt][2 * h], scale * x.v[nt][2 * h + 1]);
      float2* q = reinterpret_cast<float2*>(p + (g + 8 * h) * 16 + 8 * nt + 2 * t);
      if (STREAM) __stcs(q, v);
      else *q = v;
    }
}
// x = P^T of the row-major 16 x 16 at p (strided reads of rows usually just loaded: L1 hits)
__device__ __forceinline__ void f_load_t(F16& x, const float* __restrict__ p, int lane) {
#pragma unroll
  for (int n2 = 0; n2 < 2; ++n2)
#pragma unroll
    for (int q = 0; q < 4; ++q) x.v[n2][q] = __ldg(p + fcol(lane, n2, q) * 16 + frow(lane, q));
}

// p[c][r] = x[r][c]
__device__ __forceinline__ void f_store_t(float* p, const F16& x, int lane) {
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) p[fcol(lane, nt, e) * 16 + frow(lane, e)] = x.v[nt][e];
}
__device__ __forceinline__ void f_axpy(F16& y, float a, const F16& x) {
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) y.v[nt][e] = fmaf(a, x.v[nt][e], y.v[nt][e]);
}
__device__ __forceinline__ float f_dot(const F16& x, const F16& y) {
  float s = 0.0f;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) s = fmaf(x.v[nt][e], y.v[nt][e], s);
  return s;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(FULL, v, off);
  return v;
}

// --------------------------------------------- fp64 fragments (recurrent products)
// F16D holds the same matrix entries as F16 (same lane and slot), in fp64.
struct F16D {
  double v[2][4];
};

// d (8 x 8) += A (8 x 4) * B (4 x 8), fp64 in and out.  Lane (g, t): a = A[g][t],
// b = B[t][g], d = D[g][2 t], D[g][2 t + 1].
__device__ __forceinline__ void dmma(double (&d)[2], double a, double b) {
  asm("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0,%1}, {%2}, {%3}, {%0,%1};\n"
      : "+d"(d[0]), "+d"(d[1])
      : "d"(a), "d"(b));
}

// A B^T on fp64 fragments.  Output tile (h, nz) = rows 8 h.., columns 8 nz..; its four
// k-steps of 4 take, in slot t, the column 8 nt + 2 t + c (k-step 2 nt + c) of the rows
// of A and of B that the lane holds -- the same column permutation on both sides.
__device__ __forceinline__ F16D nt64(const F16D& A, const F16D& B) {
  F16D z;
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int nz = 0; nz < 2; ++nz) {
      double d[2] = {0.0, 0.0};
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int c = 0; c < 2; ++c) dmma(d, A.v[nt][2 * h + c], B.v[nt][2 * nz + c]);
      z.v[nz][2 * h] = d[0];
      z.v[nz][2 * h + 1] = d[1];
    }
  return z;
}

__device__ __forceinline__ F16D to_d(const F16& x) {
  F16D y;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) y.v[nt][e] = (double)x.v[nt][e];
  return y;
}
__device__ __forceinline__ F16 to_f(const F16D& x) {
  F16 y;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) y.v[nt][e] = __double2float_rn(x.v[nt][e]);
  return y;
}
__device__ __forceinline__ void d_zero(F16D& x) {
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) x.v[nt][e] = 0.0;
}
__device__ __forceinline__ F16D d_identity(int lane) {
  F16D x;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) x.v[nt][e] = (frow(lane, e) == fcol(lane, nt, e)) ? 1.0 : 0.0;
  return x;
}
// y += a x (x fp32)
__device__ __forceinline__ void d_axpy(F16D& y, float a, const F16& x) {
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) y.v[nt][e] = fma((double)a, (double)x.v[nt][e], y.v[nt][e]);
}
__device__ __forceinline__ F16D transpose64(const F16D& X, int lane) {
  F16D z;
  transpose_tiles(z.v, X.v, lane);
  return z;
}

// In-place Gauss-Jordan inverse of the fragment in deviation form (as gj_inverse_dev in
// csn_common.cuh): on entry E = A - I for A = I - Omega (no pivoting: Omega skew, pivots
// >= 1), on exit E = A^{-1} - I, so entries near 1 are carried as their deviations.
// Pivot k: row k lives in the quad g = k % 8, column k in the lanes t = (k % 8) / 2.  With
// d = 1 + E_kk, u = column k of E and v = row k of E except v_k = E_kk + 2, the whole
// in-place step
//   E_ij - E_ik E_kj / d,  E_kj / d (row k),  -E_ik / d (column k),  -E_kk / d (pivot)
// is the single rank-1 update E <- E - u v^T / d.
__device__ __forceinline__ void gj_inverse_dev(F16& A, int lane) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const int kh = k >> 3, kg = k & 7;                   // row k = kg + 8 kh
    const int kn = k >> 3, kt = (k & 7) >> 1, ke = k & 1;  // col k = 8 kn + 2 kt + ke
    float v[2][2], u[2];
#pragma unroll
    for (int n2 = 0; n2 < 2; ++n2)
#pragma unroll
      for (int c = 0; c < 2; ++c) v[n2][c] = __shfl_sync(FULL, A.v[n2][2 * kh + c], 4 * kg + t);
#pragma unroll
    for (int h = 0; h < 2; ++h) u[h] = __shfl_sync(FULL, A.v[kn][2 * h + ke], 4 * g + kt);
    const float piv = __shfl_sync(FULL, A.v[kn][2 * kh + ke], 4 * kg + kt);
    const float inv = __frcp_rn(1.0f + piv);
    if (t == kt) v[kn][ke] += 2.0f;  // this lane holds column k
    const float p0 = u[0] * inv, p1 = u[1] * inv;
#pragma unroll
    for (int n2 = 0; n2 < 2; ++n2)
#pragma unroll
      for (int e = 0; e < 4; ++e) A.v[n2][e] = fmaf(-((e >> 1) ? p1 : p0), v[n2][e & 1], A.v[n2][e]);
  }
}

// ------------------------------------------------------------- rotor generators
// Each lane's 8 entries of Omega are sums of up to NTERM signed generators; the terms
// are packed once per kernel as bytes (bits 0-6 generator index, bit 7 negative; index
// K points at a zero slot).
struct BlockTab {
  unsigned char col[CSN_CL8_NBIV][16];
  signed char sgn[CSN_CL8_NBIV][16];
};

template <int BASIS>
struct NTerms {
  static constexpr int value = (BASIS == BASIS_TRIU) ? 1 : 3;
};

__device__ __forceinline__ int triu_index(int i, int j) { return i * (2 * D - i - 1) / 2 + (j - i - 1); }

template <int BASIS, int K>
__device__ __forceinline__ void make_terms(uint32_t (&terms)[2][4], const BlockTab& tab, int lane) {
#pragma unroll
  for (int n2 = 0; n2 < 2; ++n2)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int r = frow(lane, e), c = fcol(lane, n2, e);
      uint32_t packed = (uint32_t)K | ((uint32_t)K << 8) | ((uint32_t)K << 16);
      if constexpr (BASIS == BASIS_TRIU) {
        if (r < c) packed = (packed & ~0xffu) | (uint32_t)triu_index(r, c);
        else if (r > c) packed = (packed & ~0xffu) | (uint32_t)triu_index(c, r) | 0x80u;
      } else {
        // GA: byte offsets into the signed staging gs[0, 2K] = (g, 0, -g), so a term is one
        // load and one add; 4 (2K) < 256 for K = 28
        static_assert(4 * (2 * K) < 256, "GA term offsets must fit a byte");
        packed = (uint32_t)(4 * K) * 0x010101u;
        int m = 0;
        for (int k = 0; k < K; ++k) {
          if (tab.col[k][r] == c && m < 3) {
            const uint32_t byte = 4u * (uint32_t)(tab.sgn[k][r] < 0 ? K + 1 + k : k);
            packed = (packed & ~(0xffu << (8 * m))) | (byte << (8 * m));
            ++m;
          }
        }
      }
      terms[n2][e] = packed;
    }
}

// Om = h Omega from the generators in shared memory (gs[K] == 0; for the GA basis also
// gs[K + 1 + k] = -g_k, and the terms are byte offsets).
template <int BASIS>
__device__ __forceinline__ void build_Om(F16& Om, const float* gs, const uint32_t (&terms)[2][4], float h) {
#pragma unroll
  for (int n2 = 0; n2 < 2; ++n2)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float om = 0.0f;
      if constexpr (BASIS == BASIS_TRIU) {
        const uint32_t byte = terms[n2][e] & 0xffu;
        const float v = gs[byte & 0x7fu];
        om = (byte & 0x80u) ? -v : v;
      } else {
        const char* gb = reinterpret_cast<const char*>(gs);
#pragma unroll
        for (int m = 0; m < NTerms<BASIS>::value; ++m)
          om += *reinterpret_cast<const float*>(gb + ((terms[n2][e] >> (8 * m)) & 0xffu));
      }
      Om.v[n2][e] = h * om;
    }
}

// |Om|_F^2 at or below this takes the series (|Om|_2 <= |Om|_F <= 0.05).
constexpr float kSeriesFro2 = 0.0025f;

// M = sa (2 (I - Om)^{-1} - I) = sa (I + 2 E) with E = (I - Om)^{-1} - I, in place on Om.
// Both ways keep E small until M is formed, so no entry near 1 of (I - Om)^{-1} is rounded
// on its own (that rounding leaves every rotor short of orthogonal in the same direction,
// which an undamped scan compounds over the whole sequence):
//  * |Om|_F <= 0.05: E = Om (I - Om)^{-1} = A + A P' with A = Om + W, W = Om^2 (symmetric),
//    P' = W + W^2 + W W^2 -- the series of (I - W)^{-1} to W^3 (truncation eps^8 / (1 - eps^2)
//    <= 4e-11) -- four NT products (tf32 MMAs) of matrices of size eps^2 or less, so their
//    truncating accumulation is far below fp32 rounding of E.  W, W^2 and A P' are 3xTF32;
//    W^3 <= eps^6 <= 1.6e-8 is a single TF32 product (error <= 2^-10 of it, under 0.1 ulp of
//    P' ~ eps^2);
//  * larger Om: Gauss-Jordan elimination in deviation form (round-to-nearest FMAs).
// The choice is uniform across the warp (one matrix per warp).
__device__ __forceinline__ void cayley(F16& M, float sa, int lane) {
  const float fro2 = warp_sum(f_dot(M, M));
  if (fro2 <= kSeriesFro2) {
    F16S Os;
    split(Os, M);
    F16 W;
    nt(W, Os, Os);  // Om Om^T = -Om^2
#pragma unroll
    for (int n2 = 0; n2 < 2; ++n2)
#pragma unroll
      for (int e = 0; e < 4; ++e) W.v[n2][e] = -W.v[n2][e];
    F16S Ws;
    split(Ws, W);
    F16 W2;
    nt(W2, Ws, Ws);  // W W^T = W^2
    F16 W3;
    nt_head(W3, Ws, W2);  // W (W^2)^T = W^3
    F16 A, Pp;
#pragma unroll
    for (int n2 = 0; n2 < 2; ++n2)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        A.v[n2][e] = M.v[n2][e] + W.v[n2][e];
        Pp.v[n2][e] = (W.v[n2][e] + W2.v[n2][e]) + W3.v[n2][e];
      }
    F16S As, Ps;
    split(As, A);
    split(Ps, Pp);
    F16 AP;
    nt(AP, As, Ps);  // A P'^T = A P' (P' symmetric)
#pragma unroll
    for (int n2 = 0; n2 < 2; ++n2)
#pragma unroll
      for (int e = 0; e < 4; ++e) M.v[n2][e] = A.v[n2][e] + AP.v[n2][e];
  } else {
#pragma unroll
    for (int n2 = 0; n2 < 2; ++n2)
#pragma unroll
      for (int e = 0; e < 4; ++e) M.v[n2][e] = -M.v[n2][e];  // E = (I - Om) - I
    gj_inverse_dev(M, lane);
  }
#pragma unroll
  for (int n2 = 0; n2 < 2; ++n2)
#pragma unroll
    for (int e = 0; e < 4; ++e)
      M.v[n2][e] = sa * fmaf(2.0f, M.v[n2][e], (frow(lane, e) == fcol(lane, n2, e)) ? 1.0f : 0.0f);
}

__device__ const Cl8BivTab g_cl8_tab = cl8_biv_tab();

__device__ __forceinline__ void load_tab(BlockTab& tab) {
  for (int i = threadIdx.x; i < CSN_CL8_NBIV * 16; i += blockDim.x) {
    tab.col[i / 16][i % 16] = g_cl8_tab.col[i / 16][i % 16];
    tab.sgn[i / 16][i % 16] = g_cl8_tab.sgn[i / 16][i % 16];
  }
}

// Per-warp step context: coordinates, the generator slot and the packed Omega terms.
struct Warp {
  int lane;
  int64_t b, n, j, s, t0, t1;
  float* gs;  // K + 1 floats of this warp (gs[K] = 0), 2K + 1 for the GA basis (then -g)
  float* zs;  // 16 x ZST dOmega scratch (backward apply)
};

#define S16_PROLOGUE(BASIS, K)                                                   \
  __shared__ __align__(16) float sm_g[WARPS][128];                               \
  __shared__ __align__(16) float sm_z[WARPS][16 * ZST];                          \
  __shared__ BlockTab tab;                                                       \
  if (BASIS == BASIS_GA) load_tab(tab);                                          \
  __syncthreads();                                                               \
  const int wi = threadIdx.x >> 5;                                               \
  const int64_t wid = blockIdx.x * (int64_t)WARPS + wi;                          \
  if (wid >= a.B * a.N * a.nchunks) return;                                      \
  Warp w;                                                                        \
  w.lane = threadIdx.x & 31;                                                     \
  w.n = wid % a.N;                                                               \
  w.j = (wid / a.N) % a.nchunks;                                                 \
  w.b = wid / (a.N * a.nchunks);                                                 \
  w.s = w.b * a.N + w.n;                                                         \
  w.t0 = w.j * a.chunk;                                                          \
  w.t1 = min(a.T, w.t0 + a.chunk);                                               \
  w.gs = sm_g[wi];                                                               \
  w.zs = sm_z[wi];                                                               \
  uint32_t terms[2][4] = {{0u, 0u, 0u, 0u}, {0u, 0u, 0u, 0u}};                   \
  if (SRC == SRC_ROTOR) {                                                        \
    make_terms<BASIS, K>(terms, tab, w.lane);                                    \
    if (w.lane == 0) w.gs[K] = 0.0f;                                             \
  }

// Generators of element e into registers (lane holds k = lane + 32 m).
template <int K>
__device__ __forceinline__ void fetch_gens(float (&gr)[(K + 31) / 32], const float* __restrict__ gens,
                                           int64_t e, int lane) {
#pragma unroll
  for (int m = 0; m < (K + 31) / 32; ++m) {
    const int k = lane + 32 * m;
    gr[m] = (k < K) ? __ldg(gens + e * K + k) : 0.0f;
  }
}
// NEG: also -g at gs[K + 1 + k], for the GA-basis Omega of a pass that builds rotors.
template <int K, bool NEG>
__device__ __forceinline__ void stage_gens(float* gs, const float (&gr)[(K + 31) / 32], int lane) {
  __syncwarp();  // previous step's readers are done
#pragma unroll
  for (int m = 0; m < (K + 31) / 32; ++m) {
    const int k = lane + 32 * m;
    if (k < K) {
      gs[k] = gr[m];
      if constexpr (NEG) gs[K + 1 + k] = -gr[m];
    }
  }
  __syncwarp();
}

// dt, gamma and the decay scalars of element e at time t (the rotor itself comes from the cache).
template <bool DAMPED>
__device__ __forceinline__ void rotor_scalars(const ScanArgs& a, const Warp& w, int64_t e, int64_t t,
                                              float& alpha, float& sa, float& dtv, float& gam) {
  dtv = __ldg(a.dt + dt_index(a, w.b, tphys(a, t), w.n));
  if constexpr (DAMPED) {
    gam = __ldg(a.gamma + e);
    alpha = 1.0f / (1.0f + expf(gam * dtv));
    sa = sqrtf(alpha);
  } else {
    gam = 0.0f;
    alpha = sa = 1.0f;
  }
}

// The step matrix M (Cayley rotor or a given M) of element e at time t.
// CIN: the rotors come from the cache a.Mc_in (a compile-time choice, so the kernels that
// load them carry none of the registers of the rotor build).
template <int SRC, int BASIS, bool DAMPED, int K, bool CIN>
__device__ __forceinline__ void step_matrix(const ScanArgs& a, const Warp& w, const uint32_t (&terms)[2][4],
                                            int64_t e, int64_t t, F16& M, float& alpha, float& sa,
                                            float& dtv, float& gam) {
  if constexpr (SRC == SRC_MC) {
    f_load(M, a.M + e * DD, w.lane);
    alpha = sa = 1.0f;
    dtv = gam = 0.0f;
  } else {
    dtv = __ldg(a.dt + dt_index(a, w.b, tphys(a, t), w.n));
    if constexpr (DAMPED) {
      gam = __ldg(a.gamma + e);
      alpha = 1.0f / (1.0f + expf(gam * dtv));
      sa = sqrtf(alpha);
    } else {
      gam = 0.0f;
      alpha = sa = 1.0f;
    }
    if constexpr (CIN) {
      f_load(M, a.Mc_in + e * DD, w.lane);  // cached rotor of this step
    } else {
      build_Om<BASIS>(M, w.gs, terms, 0.5f * dtv);
      cayley(M, sa, w.lane);
      if (a.Mc_out) f_store<false>(a.Mc_out + e * DD, M, w.lane);
    }
  }
}

// ---------------------------------------------------------------------- forward
// REDUCE: chunk aggregate (P = M_last ... M_first, c = chunk scanned from zero);
// otherwise the apply pass from the chunk's carry.
template <bool REDUCE, int SRC, int BASIS, bool DAMPED, bool TWO, bool CIN>
__global__ void __launch_bounds__(128, 3) fwd16_kernel(ScanArgs a) {
  constexpr int K = GenCount<16, BASIS>::K;
  constexpr int KR = (K + 31) / 32;
  S16_PROLOGUE(BASIS, K);
  const int lane = w.lane;
  F16D X, Pt;  // recurrent: fp64 fragments
  if (REDUCE) {
    d_zero(X);
    Pt = d_identity(lane);
  } else if (a.nchunks > 1) {
    F16 x;
    f_load_plain(x, a.carry + (w.s * a.nchunks + w.j) * DD, lane);
    X = to_d(x);
  } else if (a.h0) {
    F16 x;
    f_load(x, a.h0 + w.s * DD, lane);
    X = to_d(x);
  } else {
    d_zero(X);
  }
  float gr[KR];
  if (SRC == SRC_ROTOR && !CIN && w.t0 < w.t1) fetch_gens<K>(gr, a.gens, elem(a, w.b, w.t0, w.n), lane);
  // cached rotors: the next step's rotor and injection are loaded a step ahead
  F16 Mn, Cn;
  if constexpr (CIN) {
    if (w.t0 < w.t1) {
      const int64_t e0 = elem(a, w.b, w.t0, w.n);
      f_load(Mn, a.Mc_in + e0 * DD, lane);
      f_load(Cn, a.S + e0 * DD, lane);
    }
  }
  for (int64_t t = w.t0; t < w.t1; ++t) {
    const int64_t e = elem(a, w.b, t, w.n);
    F16 Cin, M;
    float alpha, sa, dtv, gam;
    if constexpr (CIN) {
      Cin = Cn;
      M = Mn;
      if (t + 1 < w.t1) {
        const int64_t e1 = elem(a, w.b, t + 1, w.n);
        f_load(Mn, a.Mc_in + e1 * DD, lane);
        f_load(Cn, a.S + e1 * DD, lane);
      }
      rotor_scalars<DAMPED>(a, w, e, t, alpha, sa, dtv, gam);
    } else {
      f_load(Cin, (SRC == SRC_MC ? a.C : a.S) + e * DD, lane);
      if constexpr (SRC == SRC_ROTOR) {
        stage_gens<K, BASIS == BASIS_GA && !CIN>(w.gs, gr, lane);
        if (t + 1 < w.t1) fetch_gens<K>(gr, a.gens, elem(a, w.b, t + 1, w.n), lane);
      }
      step_matrix<SRC, BASIS, DAMPED, K, CIN>(a, w, terms, e, t, M, alpha, sa, dtv, gam);
    }
    const float cs = (SRC == SRC_ROTOR && DAMPED) ? (1.0f - alpha) : 1.0f;
    const F16D Md = to_d(M);
    F16D V;
    if constexpr (TWO) {
      V = nt64(Md, X);  // M X^T
    } else {
      V = transpose64(X, lane);  // X^T
    }
    X = nt64(Md, V);  // M V^T:  M X M^T  |  M X
    d_axpy(X, cs, Cin);
    if constexpr (REDUCE) {
      Pt = nt64(Pt, Md);  // P^T M^T = (M P)^T
    } else {
      f_store<true>(a.out + e * DD, to_f(X), lane);
    }
  }
  if constexpr (REDUCE) {
    f_store<false>(a.aggC + (w.s * a.nchunks + w.j) * DD, to_f(X), lane);
    f_store_t(a.aggP + (w.s * a.nchunks + w.j) * DD, to_f(Pt), lane);
  }
}

// ------------------------------------------------------------- backward: reduce
// c' = gradient leaving the chunk at its first step with zero gradient from the right,
// P = M_last ... M_first (built as P <- P M walking backwards).
template <int SRC, int BASIS, bool DAMPED, bool TWO, bool CIN>
__global__ void __launch_bounds__(128, 4) bwd16_reduce_kernel(ScanArgs a) {
  constexpr int K = GenCount<16, BASIS>::K;
  constexpr int KR = (K + 31) / 32;
  S16_PROLOGUE(BASIS, K);
  if (w.j == 0 && !a.agg_mode) return;  // chunk 0's aggregate is only used by shard aggregates
  const int lane = w.lane;
  F16D Gc, P;  // recurrent: fp64 fragments
  d_zero(Gc);
  P = d_identity(lane);
  float gr[KR];
  if (SRC == SRC_ROTOR && !CIN && w.t0 < w.t1) fetch_gens<K>(gr, a.gens, elem(a, w.b, w.t1 - 1, w.n), lane);
  // cached rotors: the next step's M^T (read transposed from the cache) and dX a step ahead
  F16 Mtn, dXn;
  if constexpr (CIN) {
    if (w.t0 < w.t1) {
      const int64_t e0 = elem(a, w.b, w.t1 - 1, w.n);
      f_load_t(Mtn, a.Mc_in + e0 * DD, lane);
      f_load(dXn, a.dX + e0 * DD, lane);
    }
  }
  for (int64_t t = w.t1 - 1; t >= w.t0; --t) {
    const int64_t e = elem(a, w.b, t, w.n);
    F16 dX, Mt;
    if constexpr (CIN) {
      dX = dXn;
      Mt = Mtn;
      if (t - 1 >= w.t0) {
        const int64_t e1 = elem(a, w.b, t - 1, w.n);
        f_load_t(Mtn, a.Mc_in + e1 * DD, lane);
        f_load(dXn, a.dX + e1 * DD, lane);
      }
    } else {
      f_load(dX, a.dX + e * DD, lane);
      if constexpr (SRC == SRC_ROTOR) {
        stage_gens<K, BASIS == BASIS_GA && !CIN>(w.gs, gr, lane);
        if (t - 1 >= w.t0) fetch_gens<K>(gr, a.gens, elem(a, w.b, t - 1, w.n), lane);
      }
      F16 M;
      float alpha, sa, dtv, gam;
      step_matrix<SRC, BASIS, DAMPED, K, CIN>(a, w, terms, e, t, M, alpha, sa, dtv, gam);
      // M in memory (a given M): read it transposed instead of a product
      if (SRC == SRC_MC) {
        f_load_t(Mt, a.M + e * DD, lane);
      } else {
        transpose(Mt, M, lane);
      }
    }
    const F16D Mtd = to_d(Mt);
    d_axpy(Gc, 1.0f, dX);  // G = g + dX
    F16D W;
    if constexpr (TWO) {
      W = nt64(Mtd, Gc);  // M^T G^T
    } else {
      W = transpose64(Gc, lane);  // G^T
    }
    Gc = nt64(Mtd, W);  // M^T G M  |  M^T G
    if (!a.reuse_P) P = nt64(P, Mtd);  // P M
  }
  f_store<false>(a.aggC + (w.s * a.nchunks + w.j) * DD, to_f(Gc), lane);
  if (!a.reuse_P) f_store<false>(a.aggP + (w.s * a.nchunks + w.j) * DD, to_f(P), lane);
}

// -------------------------------------------------------------- backward: apply
// Per step t (reverse):  G = H + dX_t,  dC = G (rotor: dS = (1 - a) G)
//   dM = G M Xp^T + G^T M Xp  (one-sided: G Xp^T),  Xp = X_{t-1}
//   rotor: da = -<G, S> + <dM, M> / (2 a);  dOmega = 0.5 sa B dM B with B = I + M^T / sa;
//          dg_k = <dOmega, E_k> dt / 2
//   H <- M^T G M  (one-sided: M^T G)
template <int SRC, int BASIS, bool DAMPED, bool TWO, bool CIN>
__global__ void __launch_bounds__(128, 3) bwd16_apply_kernel(ScanArgs a) {
  constexpr int K = GenCount<16, BASIS>::K;
  constexpr int KR = (K + 31) / 32;
  S16_PROLOGUE(BASIS, K);
  const int lane = w.lane;
  F16D H;  // recurrent gradient carry: fp64 fragment
  {
    F16 h;
    if (a.nchunks > 1) f_load_plain(h, a.carry + (w.s * a.nchunks + w.j) * DD, lane);
    else if (a.hT) f_load(h, a.hT + w.s * DD, lane);
    else f_zero(h);
    H = to_d(h);
  }
  // triu generator k = lane + 32 m  ->  (i, j) packed as i * 16 + j
  int kpair[KR];
  if constexpr (SRC == SRC_ROTOR && BASIS == BASIS_TRIU) {
#pragma unroll
    for (int m = 0; m < KR; ++m) {
      int k = lane + 32 * m, u = 0;
      if (k < K) {
        while (k >= D - 1 - u) { k -= D - 1 - u; ++u; }
        kpair[m] = u * 16 + (u + 1 + k);
      } else {
        kpair[m] = 0;
      }
    }
  }
  float gr[KR];
  if (SRC == SRC_ROTOR && w.t0 < w.t1) fetch_gens<K>(gr, a.gens, elem(a, w.b, w.t1 - 1, w.n), lane);
  for (int64_t t = w.t1 - 1; t >= w.t0; --t) {
    const int64_t e = elem(a, w.b, t, w.n);
    F16 dX, Xp, Sx;
    f_load(dX, a.dX + e * DD, lane);
    const float* xprev = (t > 0) ? (a.X + elem(a, w.b, t - 1, w.n) * DD) : (a.h0 ? a.h0 + w.s * DD : nullptr);
    if (xprev) f_load(Xp, xprev, lane);
    if (SRC == SRC_ROTOR && DAMPED) f_load(Sx, a.S + e * DD, lane);
    if constexpr (SRC == SRC_ROTOR) {
      stage_gens<K, BASIS == BASIS_GA && !CIN>(w.gs, gr, lane);
      if (t - 1 >= w.t0) fetch_gens<K>(gr, a.gens, elem(a, w.b, t - 1, w.n), lane);
    }
    F16 M;
    float alpha, sa, dtv, gam;
    step_matrix<SRC, BASIS, DAMPED, K, CIN>(a, w, terms, e, t, M, alpha, sa, dtv, gam);
    F16S Ms, Mts;
    split(Ms, M);
    F16 Mt;
    transpose(Mt, M, lane);
    split(Mts, Mt);
    // G = H + dX in fp64; the carry to the previous step, M^T G M (one-sided M^T G), is
    // formed from it right away, and the step's gradients use G rounded to fp32
    F16 G;
    {
      F16D Gd = H;
      d_axpy(Gd, 1.0f, dX);
      G = to_f(Gd);
      const F16D Mtd = to_d(Mt);
      if constexpr (TWO) {
        H = nt64(Mtd, nt64(Mtd, Gd));  // M^T (M^T G^T)^T = M^T G M
      } else {
        H = nt64(Mtd, transpose64(Gd, lane));  // M^T G
      }
    }
    F16S Gs;
    split(Gs, G);
    const float cs = (SRC == SRC_ROTOR && DAMPED) ? (1.0f - alpha) : 1.0f;
    f_store<true>(a.dC + e * DD, G, lane, cs);  // dC | dS
    // ---- dM
    F16 dM;
    F16 Gt;  // G^T (two-sided dM, one-sided carry)
    transpose(Gt, G, lane);
    F16S Gts;
    split(Gts, Gt);
    if (xprev) {
      F16S Xps;
      split(Xps, Xp);
      if constexpr (TWO) {
        F16 GM;
        nt(GM, Gs, Mts);  // G M
        F16S GMs;
        split(GMs, GM);
        nt(dM, GMs, Xps);  // G M Xp^T
        F16 Xpt;  // X_{t-1}^T straight from memory (the rows were just loaded: L1 hits)
#pragma unroll
        for (int n2 = 0; n2 < 2; ++n2)
#pragma unroll
          for (int q = 0; q < 4; ++q) Xpt.v[n2][q] = __ldg(xprev + fcol(lane, n2, q) * 16 + frow(lane, q));
        F16S Xpts;
        split(Xpts, Xpt);
        F16 XM;
        nt(XM, Xpts, Ms);  // Xp^T M^T
        F16S XMs;
        split(XMs, XM);
        F16 T2;
        nt(T2, Gts, XMs);  // G^T M Xp
        f_axpy(dM, 1.0f, T2);
      } else {
        nt(dM, Gs, Xps);  // G Xp^T
      }
    } else {
      f_zero(dM);
    }
    if constexpr (SRC == SRC_MC) {
      f_store<true>(a.dM + e * DD, dM, lane);
    } else {
      float da = 0.0f;
      if constexpr (DAMPED) {
        const float p1 = warp_sum(f_dot(dM, M));
        const float p2 = warp_sum(f_dot(G, Sx));
        da = -p2 + p1 / (2.0f * alpha);
      }
      // dOmega^T = 0.5 sa Bt dM^T Bt,  Bt = B^T = I + M / sa
      const float inv_sa = 1.0f / sa;
      F16 Zt;
      F16S dMs;
      split(dMs, dM);
      if constexpr (!DAMPED) {
        // as Y = Bt dM^T = dM^T + (M dM^T) / sa and Zt = Y Bt = Y + (Y M) / sa: the identity
        // parts are exact additions and the products reuse the split M and M^T
        F16 Y, dMt;
        nt(Y, Ms, dMs);  // M dM^T
        transpose(dMt, dM, lane);
#pragma unroll
        for (int n2 = 0; n2 < 2; ++n2)
#pragma unroll
          for (int q = 0; q < 4; ++q) Y.v[n2][q] = fmaf(Y.v[n2][q], inv_sa, dMt.v[n2][q]);
        F16S Ys;
        split(Ys, Y);
        nt(Zt, Ys, Mts);  // Y M
#pragma unroll
        for (int n2 = 0; n2 < 2; ++n2)
#pragma unroll
          for (int q = 0; q < 4; ++q) Zt.v[n2][q] = fmaf(Zt.v[n2][q], inv_sa, Y.v[n2][q]);
      } else {
        // with the decay's live values the reuse above spills: B and B^T built and split
        F16 Bt, Bm;
#pragma unroll
        for (int n2 = 0; n2 < 2; ++n2)
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float id = (frow(lane, q) == fcol(lane, n2, q)) ? 1.0f : 0.0f;
            Bt.v[n2][q] = fmaf(M.v[n2][q], inv_sa, id);
            Bm.v[n2][q] = fmaf(Mt.v[n2][q], inv_sa, id);
          }
        F16S Bts, Bms;
        split(Bts, Bt);
        split(Bms, Bm);
        F16 Y;
        nt(Y, Bts, dMs);  // Bt dM^T
        F16S Ys;
        split(Ys, Y);
        nt(Zt, Ys, Bms);  // Bt dM^T Bt
      }
      // dOmega[u][v] = 0.5 sa Zt[v][u] -> zs[u * ZST + v]
      __syncwarp();
#pragma unroll
      for (int n2 = 0; n2 < 2; ++n2)
#pragma unroll
        for (int q = 0; q < 4; ++q)
          w.zs[fcol(lane, n2, q) * ZST + frow(lane, q)] = 0.5f * sa * Zt.v[n2][q];
      __syncwarp();
      float ddt = 0.0f;
      const float hdt = 0.5f * dtv;
#pragma unroll
      for (int m = 0; m < KR; ++m) {
        const int k = lane + 32 * m;
        if (k < K) {
          float pk;
          if constexpr (BASIS == BASIS_TRIU) {
            const int u = kpair[m] >> 4, v = kpair[m] & 15;
            pk = w.zs[u * ZST + v] - w.zs[v * ZST + u];
          } else {
            pk = 0.0f;
#pragma unroll
            for (int u = 0; u < 16; ++u) pk = fmaf((float)tab.sgn[k][u], w.zs[u * ZST + tab.col[k][u]], pk);
          }
          a.dgens[e * K + k] = pk * hdt;
          ddt = fmaf(pk, 0.5f * w.gs[k], ddt);
        }
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
  }
  if (w.j == 0 && a.dh0) f_store<false>(a.dh0 + w.s * DD, to_f(H), lane);
}

unsigned nblk(int64_t warps) { return (unsigned)((warps + WARPS - 1) / WARPS); }

// Launch a pass in its rotor-cache-loading form when a.Mc_in is set (rotor sources only).
template <bool REDUCE, int SRC, int BASIS, bool DAMPED, bool TWO>
void launch_fwd16(const ScanArgs& a, unsigned grid, cudaStream_t st) {
  if constexpr (SRC == SRC_ROTOR) {
    if (a.Mc_in) {
      fwd16_kernel<REDUCE, SRC, BASIS, DAMPED, TWO, true><<<grid, 128, 0, st>>>(a);
      return;
    }
  }
  fwd16_kernel<REDUCE, SRC, BASIS, DAMPED, TWO, false><<<grid, 128, 0, st>>>(a);
}
template <int SRC, int BASIS, bool DAMPED, bool TWO>
void launch_bwd16_reduce(const ScanArgs& a, unsigned grid, cudaStream_t st) {
  if constexpr (SRC == SRC_ROTOR) {
    if (a.Mc_in) {
      bwd16_reduce_kernel<SRC, BASIS, DAMPED, TWO, true><<<grid, 128, 0, st>>>(a);
      return;
    }
  }
  bwd16_reduce_kernel<SRC, BASIS, DAMPED, TWO, false><<<grid, 128, 0, st>>>(a);
}
template <int SRC, int BASIS, bool DAMPED, bool TWO>
void launch_bwd16_apply(const ScanArgs& a, unsigned grid, cudaStream_t st) {
  if constexpr (SRC == SRC_ROTOR) {
    if (a.Mc_in) {
      bwd16_apply_kernel<SRC, BASIS, DAMPED, TWO, true><<<grid, 128, 0, st>>>(a);
      return;
    }
  }
  bwd16_apply_kernel<SRC, BASIS, DAMPED, TWO, false><<<grid, 128, 0, st>>>(a);
}

template <int SRC, int BASIS, bool DAMPED, bool TWO>
int run16(const ScanArgs& a, bool bwd, cudaStream_t st) {
  const int64_t S = a.B * a.N;
  const int64_t total = S * a.nchunks;
  if (a.agg_mode == 1) {
    if (total == 0) return CSN_OK;
    if (!bwd) {
      {
        KernelTimer kt("agg_fwd_reduce", st);
        launch_fwd16<true, SRC, BASIS, DAMPED, TWO>(a, nblk(total), st);
      }
      KernelTimer kt("agg_compose", st);
      compose_kernel<16, TWO, false><<<nblk(S), 128, 0, st>>>(a);
    } else {
      {
        KernelTimer kt("agg_bwd_reduce", st);
        launch_bwd16_reduce<SRC, BASIS, DAMPED, TWO>(a, nblk(total), st);
      }
      KernelTimer kt("agg_compose", st);
      compose_kernel<16, TWO, true><<<nblk(S), 128, 0, st>>>(a);
    }
    return check_launch("shard aggregate (D=16)");
  }
  if (!bwd) {
    if (total == 0) return CSN_OK;
    ScanArgs ap = a;  // apply pass: reads the rotors the reduce pass stored
    if (a.nchunks > 1) {
      if (a.agg_mode != 2) {
        KernelTimer kt("fwd_reduce", st);
        launch_fwd16<true, SRC, BASIS, DAMPED, TWO>(a, nblk(total), st);
        if (a.Mc_out) {
          ap.Mc_in = a.Mc_out;
          ap.Mc_out = nullptr;
        }
      }
      KernelTimer kt("fwd_carry", st);
      launch_grouped_carry<16, TWO, false>(a, st);
    }
    KernelTimer kt("fwd_apply", st);
    launch_fwd16<false, SRC, BASIS, DAMPED, TWO>(ap, nblk(total), st);
    return check_launch("scan forward (D=16)");
  }
  if (total > 0) {
    if (a.nchunks > 1) {
      if (a.agg_mode != 2) {
        KernelTimer kt("bwd_reduce", st);
        launch_bwd16_reduce<SRC, BASIS, DAMPED, TWO>(a, nblk(total), st);
      }
      KernelTimer kt("bwd_carry", st);
      launch_grouped_carry<16, TWO, true>(a, st);
    }
    KernelTimer kt("bwd_apply", st);
    launch_bwd16_apply<SRC, BASIS, DAMPED, TWO>(a, nblk(total), st);
  }
  if (SRC == SRC_ROTOR && a.B * a.T > 0) {
    const int64_t BT = a.B * a.T;
    KernelTimer kt("reduce_channels", st);
    const int64_t H = dt_heads(a);
    reduce_channels_kernel<<<(unsigned)((BT * H + 255) / 256), 256, 0, st>>>(a.ddt_part, a.ddt, BT * H,
                                                                            a.N / H);
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
