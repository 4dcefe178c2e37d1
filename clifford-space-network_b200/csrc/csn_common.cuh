// csn_common.cuh -- shared device primitives for the rotor-scan kernels (sm_100a).
//
// Small D x D matrices (D = 4, 8) live in registers as Mat<D>; every loop is fully
// unrolled so the compiler keeps them in registers.  The in-place products below
// never need a second D x D buffer: a left product X <- M X is done column by
// column and a right product X <- X M^T row by row, each column/row depending
// only on itself.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "ga_tables.h"

namespace csn {

template <int D>
struct Mat {
  float a[D][D];
};

template <int D>
__device__ __forceinline__ void mat_zero(Mat<D>& X) {
#pragma unroll
  for (int i = 0; i < D; ++i)
#pragma unroll
    for (int j = 0; j < D; ++j) X.a[i][j] = 0.0f;
}

template <int D>
__device__ __forceinline__ void mat_identity(Mat<D>& X) {
#pragma unroll
  for (int i = 0; i < D; ++i)
#pragma unroll
    for (int j = 0; j < D; ++j) X.a[i][j] = (i == j) ? 1.0f : 0.0f;
}

// X <- M X
template <int D>
__device__ __forceinline__ void lmul(const Mat<D>& M, Mat<D>& X) {
#pragma unroll
  for (int j = 0; j < D; ++j) {
    float col[D];
#pragma unroll
    for (int i = 0; i < D; ++i) {
      float s = 0.0f;
#pragma unroll
      for (int k = 0; k < D; ++k) s = fmaf(M.a[i][k], X.a[k][j], s);
      col[i] = s;
    }
#pragma unroll
    for (int i = 0; i < D; ++i) X.a[i][j] = col[i];
  }
}

// X <- M^T X
template <int D>
__device__ __forceinline__ void lmulT(const Mat<D>& M, Mat<D>& X) {
#pragma unroll
  for (int j = 0; j < D; ++j) {
    float col[D];
#pragma unroll
    for (int i = 0; i < D; ++i) {
      float s = 0.0f;
#pragma unroll
      for (int k = 0; k < D; ++k) s = fmaf(M.a[k][i], X.a[k][j], s);
      col[i] = s;
    }
#pragma unroll
    for (int i = 0; i < D; ++i) X.a[i][j] = col[i];
  }
}

// X <- X M^T
template <int D>
__device__ __forceinline__ void rmulT(Mat<D>& X, const Mat<D>& M) {
#pragma unroll
  for (int i = 0; i < D; ++i) {
    float row[D];
#pragma unroll
    for (int l = 0; l < D; ++l) {
      float s = 0.0f;
#pragma unroll
      for (int j = 0; j < D; ++j) s = fmaf(X.a[i][j], M.a[l][j], s);
      row[l] = s;
    }
#pragma unroll
    for (int l = 0; l < D; ++l) X.a[i][l] = row[l];
  }
}

// ------------------------------------------------------------ packed fp32 (sm_100a)
// fma.rn.f32x2 / mul.rn.f32x2 do two round-to-nearest fp32 operations in one instruction
// on an even/odd register pair.  The FP32 pipe's FMA rate is the same for the scalar and
// the packed form; a packed instruction takes one issue slot for two FMAs, which leaves
// the slot to the loads, shuffles and address arithmetic around the products.
__device__ __forceinline__ uint64_t f2pack(float x, float y) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(x), "f"(y));
  return r;
}
__device__ __forceinline__ float2 f2unpack(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ uint64_t f2fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2splat(float x) { return f2pack(x, x); }
// the two halves added
__device__ __forceinline__ float f2sum(uint64_t v) {
  const float2 p = f2unpack(v);
  return p.x + p.y;
}

// X <- X M
template <int D>
__device__ __forceinline__ void rmul(Mat<D>& X, const Mat<D>& M) {
#pragma unroll
  for (int i = 0; i < D; ++i) {
    float row[D];
#pragma unroll
    for (int l = 0; l < D; ++l) {
      float s = 0.0f;
#pragma unroll
      for (int j = 0; j < D; ++j) s = fmaf(X.a[i][j], M.a[j][l], s);
      row[l] = s;
    }
#pragma unroll
    for (int l = 0; l < D; ++l) X.a[i][l] = row[l];
  }
}

// Gauss-Jordan inverse of A = I + E without pivoting, in deviation form: on entry E = A - I,
// on exit E = A^{-1} - I.  Only used on A = I - Omega with Omega skew: the symmetric part of
// A and of every Schur complement of A is the identity or larger, so every pivot is >= 1 and
// no pivoting is needed.  The elimination is the plain in-place one (pivot 1 / d, row k / d,
// column k -A_ik / d, the rest A_ij - A_ik A_kj / d), written for the deviations: the
// diagonal keeps E_ii = A_ii - 1 instead of A_ii.  For the small generators of long scans the
// entries of A^{-1} near 1 then never get rounded as numbers near 1 -- their deviations are
// carried to full relative precision -- and the rotor built from them is orthogonal to
// rounding level with no bias.  Rounding those entries themselves leaves every rotor short
// of orthogonal in the same direction, which an undamped scan compounds step after step
// (8e-4 of the state after 16384 steps of so(8) generators of size 1e-4).
template <int D>
__device__ __forceinline__ void gj_inverse_dev(Mat<D>& E) {
#pragma unroll
  for (int k = 0; k < D; ++k) {
    const float ekk = E.a[k][k];
    const float inv = 1.0f / (1.0f + ekk);
#pragma unroll
    for (int j = 0; j < D; ++j) E.a[k][j] = (j == k) ? -ekk * inv : E.a[k][j] * inv;
#pragma unroll
    for (int i = 0; i < D; ++i) {
      if (i == k) continue;
      const float f = E.a[i][k];
#pragma unroll
      for (int j = 0; j < D; ++j)
        if (j != k) E.a[i][j] = fmaf(-f, E.a[k][j], E.a[i][j]);
      E.a[i][k] = -f * inv;
    }
  }
}

// Cayley rotor M = sa (2 (I - Omega)^{-1} - I) = sa (I + 2 E) from E = (I - Omega)^{-1} - I.
template <int D>
__device__ __forceinline__ void rotor_from_dev(Mat<D>& E, float sa) {
#pragma unroll
  for (int i = 0; i < D; ++i)
#pragma unroll
    for (int j = 0; j < D; ++j) E.a[i][j] = sa * fmaf(2.0f, E.a[i][j], (i == j) ? 1.0f : 0.0f);
}

// ---------------------------------------------------------------- global loads
template <int D>
__device__ __forceinline__ void load_mat(Mat<D>& X, const float* __restrict__ p) {
  static_assert((D * D) % 4 == 0, "vector loads need D*D % 4 == 0");
  const float4* q = reinterpret_cast<const float4*>(p);
#pragma unroll
  for (int v = 0; v < D * D / 4; ++v) {
    const float4 f = __ldg(q + v);
    const int e = 4 * v;
    X.a[e / D][e % D] = f.x;
    X.a[(e + 1) / D][(e + 1) % D] = f.y;
    X.a[(e + 2) / D][(e + 2) % D] = f.z;
    X.a[(e + 3) / D][(e + 3) % D] = f.w;
  }
}

template <int D>
__device__ __forceinline__ void store_mat(float* __restrict__ p, const Mat<D>& X) {
  float4* q = reinterpret_cast<float4*>(p);
#pragma unroll
  for (int v = 0; v < D * D / 4; ++v) {
    const int e = 4 * v;
    float4 f;
    f.x = X.a[e / D][e % D];
    f.y = X.a[(e + 1) / D][(e + 1) % D];
    f.z = X.a[(e + 2) / D][(e + 2) % D];
    f.w = X.a[(e + 3) / D][(e + 3) % D];
    q[v] = f;
  }
}

// Streaming store (evict-first): outputs are not re-read by this kernel, so keep
// L2 for the inputs that the apply pass reads a second time.
template <int D>
__device__ __forceinline__ void store_mat_cs(float* __restrict__ p, const Mat<D>& X) {
  float4* q = reinterpret_cast<float4*>(p);
#pragma unroll
  for (int v = 0; v < D * D / 4; ++v) {
    const int e = 4 * v;
    float4 f;
    f.x = X.a[e / D][e % D];
    f.y = X.a[(e + 1) / D][(e + 1) % D];
    f.z = X.a[(e + 2) / D][(e + 2) % D];
    f.w = X.a[(e + 3) / D][(e + 3) % D];
    __stcs(q + v, f);
  }
}

// X += s * (matrix at p)
template <int D>
__device__ __forceinline__ void add_scaled_mat(Mat<D>& X, const float* __restrict__ p, float s) {
  const float4* q = reinterpret_cast<const float4*>(p);
#pragma unroll
  for (int v = 0; v < D * D / 4; ++v) {
    const float4 f = __ldg(q + v);
    const int e = 4 * v;
    X.a[e / D][e % D] = fmaf(s, f.x, X.a[e / D][e % D]);
    X.a[(e + 1) / D][(e + 1) % D] = fmaf(s, f.y, X.a[(e + 1) / D][(e + 1) % D]);
    X.a[(e + 2) / D][(e + 2) % D] = fmaf(s, f.z, X.a[(e + 2) / D][(e + 2) % D]);
    X.a[(e + 3) / D][(e + 3) % D] = fmaf(s, f.w, X.a[(e + 3) / D][(e + 3) % D]);
  }
}

template <int D>
__device__ __forceinline__ float mat_dot_global(const Mat<D>& X, const float* __restrict__ p) {
  const float4* q = reinterpret_cast<const float4*>(p);
  float s = 0.0f;
#pragma unroll
  for (int v = 0; v < D * D / 4; ++v) {
    const float4 f = __ldg(q + v);
    const int e = 4 * v;
    s = fmaf(X.a[e / D][e % D], f.x, s);
    s = fmaf(X.a[(e + 1) / D][(e + 1) % D], f.y, s);
    s = fmaf(X.a[(e + 2) / D][(e + 2) % D], f.z, s);
    s = fmaf(X.a[(e + 3) / D][(e + 3) % D], f.w, s);
  }
  return s;
}

// ------------------------------------------------------------ async staging
// Per-thread global -> shared copies (cp.async).  Each thread stages its own inputs
// into a private shared-memory slot one step ahead of use; cp.async.wait_group makes
// the thread's own copies visible to itself, so no block barrier is needed.
__device__ __forceinline__ void cp_async16(float* smem, const float* gmem) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async4(float* smem, const float* gmem) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}
// n floats (n % 4 == 0, both pointers 16-byte aligned)
template <int NF>
__device__ __forceinline__ void cp_async_floats(float* smem, const float* gmem) {
  static_assert(NF % 4 == 0, "16-byte granules");
#pragma unroll
  for (int v = 0; v < NF / 4; ++v) cp_async16(smem + 4 * v, gmem + 4 * v);
}

// Generator layouts accepted by the fused rotor kernels.
enum Basis : int {
  BASIS_TRIU = 0,  // reference layout: g_k at torch.triu_indices(D, D, 1)[:, k]
  BASIS_GA = 1,    // GA bivector blades through rho: Cl(3,0) for D = 4, Cl(8,0) for D = 16
};

template <int D, int BASIS>
struct GenCount {
  static constexpr int K = D * (D - 1) / 2;
};
template <>
struct GenCount<4, BASIS_GA> {
  static constexpr int K = CSN_CL3_NBIV;
};
template <>
struct GenCount<16, BASIS_GA> {
  static constexpr int K = CSN_CL8_NBIV;
};

// Load the K generators of one element (K*4 bytes, 8-byte aligned at least).
template <int K>
__device__ __forceinline__ void load_gens(float (&g)[K], const float* __restrict__ p) {
  if constexpr (K % 4 == 0) {
    const float4* q = reinterpret_cast<const float4*>(p);
#pragma unroll
    for (int v = 0; v < K / 4; ++v) {
      const float4 f = __ldg(q + v);
      g[4 * v] = f.x; g[4 * v + 1] = f.y; g[4 * v + 2] = f.z; g[4 * v + 3] = f.w;
    }
  } else if constexpr (K % 2 == 0) {
    const float2* q = reinterpret_cast<const float2*>(p);
#pragma unroll
    for (int v = 0; v < K / 2; ++v) {
      const float2 f = __ldg(q + v);
      g[2 * v] = f.x; g[2 * v + 1] = f.y;
    }
  } else {
#pragma unroll
    for (int v = 0; v < K; ++v) g[v] = __ldg(p + v);
  }
}

// rho(bivector) tables of the GA layout: Cl(3,0) on R^4, Cl(8,0) on R^16.
template <int D>
__host__ __device__ constexpr auto rho_biv_tab() {
  if constexpr (D == 4) return cl3_biv_tab();
  else return cl8_biv_tab();
}

// E <- -h * sum_k g_k E_k  (h = dt / 2) = (I - Omega) - I, the deviation of A = I - Omega
// from the identity (the input of gj_inverse_dev), for the generator layout BASIS.
template <int D, int BASIS, int K>
__device__ __forceinline__ void build_neg_omega(Mat<D>& E, const float (&g)[K], float h) {
  if constexpr (BASIS == BASIS_TRIU) {
    int k = 0;
#pragma unroll
    for (int u = 0; u < D; ++u) {
      E.a[u][u] = 0.0f;
#pragma unroll
      for (int v = u + 1; v < D; ++v) {
        const float w = h * g[k];
        E.a[u][v] = -w;
        E.a[v][u] = w;
        ++k;
      }
    }
  } else {
    mat_zero(E);
    constexpr auto tab = rho_biv_tab<D>();
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const float w = h * g[k];
#pragma unroll
      for (int u = 0; u < D; ++u) {
        const int col = tab.col[k][u];
        const float sg = tab.sgn[k][u];
        E.a[u][col] = fmaf(-sg, w, E.a[u][col]);
      }
    }
  }
}

// Projection of a D x D gradient G_Omega onto the generators:
// out_k = <G_Omega, E_k>.
template <int D, int BASIS, int K>
__device__ __forceinline__ void project_generators(const Mat<D>& Gom, float (&out)[K]) {
  if constexpr (BASIS == BASIS_TRIU) {
    int k = 0;
#pragma unroll
    for (int u = 0; u < D; ++u)
#pragma unroll
      for (int v = u + 1; v < D; ++v) {
        out[k] = Gom.a[u][v] - Gom.a[v][u];
        ++k;
      }
  } else {
    constexpr auto tab = rho_biv_tab<D>();
#pragma unroll
    for (int k = 0; k < K; ++k) {
      float s = 0.0f;
#pragma unroll
      for (int u = 0; u < D; ++u) s = fmaf((float)tab.sgn[k][u], Gom.a[u][tab.col[k][u]], s);
      out[k] = s;
    }
  }
}

}  // namespace csn
