/*
 * csn_oracle.c -- CPU float64 restatement of the Clifford Space Network rotor-scan
 * hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker and the timed CPU
 * baseline.  Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * reference leg load it.  The product path (the CUDA library) never links it.
 *
 * Every routine follows one reference function (paths relative to the reference
 * project root) and is written from the mathematics, sequentially in time, in
 * float64.  Sequences (b, n) are independent and are distributed over OpenMP
 * threads.
 *
 * Tensor layout (the reference's own): element (b, t, n) of a [B, T, N, ...]
 * tensor sits at ((b*T + t)*N + n) * stride.  Matrices are D x D row-major.
 *
 * Return codes: 0 = ok, 1 = invalid argument.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_MAXD 16

/* Number of OpenMP threads for the calls that follow (a launcher may have set
 * OMP_NUM_THREADS=1 for the whole process before the library was loaded).
 * Returns the count in effect. */
int orc_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
  return omp_get_max_threads();
#else
  (void)n;
  return 1;
#endif
}

/* ------------------------------------------------------------------------ */
/* small dense helpers                                                       */
/* ------------------------------------------------------------------------ */
static void mm(int D, const double* A, const double* B, double* Cout) {
    double tmp[ORC_MAXD * ORC_MAXD];
    for (int i = 0; i < D; ++i)
        for (int j = 0; j < D; ++j) {
            double s = 0.0;
            for (int k = 0; k < D; ++k) s += A[i * D + k] * B[k * D + j];
            tmp[i * D + j] = s;
        }
    memcpy(Cout, tmp, sizeof(double) * D * D);
}
/* C = A * B^T */
static void mm_nt(int D, const double* A, const double* B, double* Cout) {
    double tmp[ORC_MAXD * ORC_MAXD];
    for (int i = 0; i < D; ++i)
        for (int j = 0; j < D; ++j) {
            double s = 0.0;
            for (int k = 0; k < D; ++k) s += A[i * D + k] * B[j * D + k];
            tmp[i * D + j] = s;
        }
    memcpy(Cout, tmp, sizeof(double) * D * D);
}
/* C = A^T * B */
static void mm_tn(int D, const double* A, const double* B, double* Cout) {
    double tmp[ORC_MAXD * ORC_MAXD];
    for (int i = 0; i < D; ++i)
        for (int j = 0; j < D; ++j) {
            double s = 0.0;
            for (int k = 0; k < D; ++k) s += A[k * D + i] * B[k * D + j];
            tmp[i * D + j] = s;
        }
    memcpy(Cout, tmp, sizeof(double) * D * D);
}
static double dot(int n, const double* a, const double* b) {
    double s = 0.0;
    for (int i = 0; i < n; ++i) s += a[i] * b[i];
    return s;
}

/* Solve A X = Bm for X (D x D right-hand sides) by LU with partial pivoting.
 * torch.linalg.solve, which the reference Cayley uses, is LU with partial
 * pivoting as well.  Returns 1 when a zero pivot shows up. */
static int solve(int D, const double* A_in, const double* Bm, double* X) {
    double A[ORC_MAXD * ORC_MAXD], R[ORC_MAXD * ORC_MAXD];
    memcpy(A, A_in, sizeof(double) * D * D);
    memcpy(R, Bm, sizeof(double) * D * D);
    for (int c = 0; c < D; ++c) {
        int p = c;
        double best = fabs(A[c * D + c]);
        for (int r = c + 1; r < D; ++r)
            if (fabs(A[r * D + c]) > best) { best = fabs(A[r * D + c]); p = r; }
        if (best == 0.0) return 1;
        if (p != c)
            for (int j = 0; j < D; ++j) {
                double t = A[c * D + j]; A[c * D + j] = A[p * D + j]; A[p * D + j] = t;
                t = R[c * D + j]; R[c * D + j] = R[p * D + j]; R[p * D + j] = t;
            }
        for (int r = c + 1; r < D; ++r) {
            double f = A[r * D + c] / A[c * D + c];
            if (f == 0.0) continue;
            for (int j = c; j < D; ++j) A[r * D + j] -= f * A[c * D + j];
            for (int j = 0; j < D; ++j) R[r * D + j] -= f * R[c * D + j];
        }
    }
    for (int c = D - 1; c >= 0; --c)
        for (int j = 0; j < D; ++j) {
            double s = R[c * D + j];
            for (int k = c + 1; k < D; ++k) s -= A[c * D + k] * R[k * D + j];
            R[c * D + j] = s / A[c * D + c];
        }
    memcpy(X, R, sizeof(double) * D * D);
    return 0;
}

static size_t off3(long b, long t, long n, long T, long N) { return (size_t)((b * T + t) * N + n); }

/* ------------------------------------------------------------------------ */
/* plain scans                                                               */
/* ------------------------------------------------------------------------ */
/*
 * Inclusive rotor scan over time.
 *   two-sided: X_t = M_t X_{t-1} M_t^T + C_t   (python/clifford_scan.py:19-85,
 *              sequential form of tests/test_scan_equivalence.py:39-49)
 *   one-sided: X_t = M_t X_{t-1} + C_t         (csn_toolkit/csn/scan.py:24-41)
 * X_{-1} = h0 (zero when h0 == NULL), so X_0 = C_0 and M_0 is unused, as in the
 * reference, which has no initial-state argument.
 */
int orc_scan_fwd(const double* M, const double* C, const double* h0, double* X,
                 long B, long T, long N, int D, int two_sided) {
    if (D < 1 || D > ORC_MAXD || B < 0 || T < 0 || N < 0) return 1;
    const long DD = (long)D * D;
#pragma omp parallel for collapse(2) schedule(static)
    for (long b = 0; b < B; ++b)
        for (long n = 0; n < N; ++n) {
            double h[ORC_MAXD * ORC_MAXD], tmp[ORC_MAXD * ORC_MAXD];
            if (h0) memcpy(h, h0 + (b * N + n) * DD, sizeof(double) * DD);
            else memset(h, 0, sizeof(double) * DD);
            for (long t = 0; t < T; ++t) {
                const size_t o = off3(b, t, n, T, N) * DD;
                mm(D, M + o, h, tmp);
                if (two_sided) mm_nt(D, tmp, M + o, tmp);
                for (long i = 0; i < DD; ++i) h[i] = tmp[i] + C[o + i];
                memcpy(X + o, h, sizeof(double) * DD);
            }
        }
    return 0;
}

/*
 * Reverse-time adjoint of orc_scan_fwd.
 *   one-sided (csn_toolkit/csn/scan.py:44-72):
 *     G_t = dX_t + M_{t+1}^T G_{t+1};  dC_t = G_t;  dM_t = G_t X_{t-1}^T
 *   two-sided (the adjoint of python/clifford_scan.py:41-85 under autograd):
 *     G_t = dX_t + M_{t+1}^T G_{t+1} M_{t+1};  dC_t = G_t;
 *     dM_t = G_t M_t X_{t-1}^T + G_t^T M_t X_{t-1}
 * X_{-1} = h0 (zero when NULL, giving dM_0 = 0 as in the reference); dh0 is the
 * carry left after t = 0 (optional output).
 */
int orc_scan_bwd(const double* M, const double* X, const double* dX, const double* h0,
                 double* dM, double* dC, double* dh0,
                 long B, long T, long N, int D, int two_sided) {
    if (D < 1 || D > ORC_MAXD || B < 0 || T < 0 || N < 0) return 1;
    const long DD = (long)D * D;
#pragma omp parallel for collapse(2) schedule(static)
    for (long b = 0; b < B; ++b)
        for (long n = 0; n < N; ++n) {
            double carry[ORC_MAXD * ORC_MAXD], G[ORC_MAXD * ORC_MAXD];
            double xp[ORC_MAXD * ORC_MAXD], t1[ORC_MAXD * ORC_MAXD], t2[ORC_MAXD * ORC_MAXD];
            memset(carry, 0, sizeof(double) * DD);
            for (long t = T - 1; t >= 0; --t) {
                const size_t o = off3(b, t, n, T, N) * DD;
                const double* Mt = M + o;
                for (long i = 0; i < DD; ++i) G[i] = dX[o + i] + carry[i];
                memcpy(dC + o, G, sizeof(double) * DD);
                if (t > 0) memcpy(xp, X + off3(b, t - 1, n, T, N) * DD, sizeof(double) * DD);
                else if (h0) memcpy(xp, h0 + (b * N + n) * DD, sizeof(double) * DD);
                else memset(xp, 0, sizeof(double) * DD);
                if (two_sided) {
                    mm(D, G, Mt, t1);        /* G M        */
                    mm_nt(D, t1, xp, t1);    /* G M X^T    */
                    mm(D, Mt, xp, t2);       /* M X        */
                    mm_tn(D, G, t2, t2);     /* G^T M X    */
                    for (long i = 0; i < DD; ++i) dM[o + i] = t1[i] + t2[i];
                    mm_tn(D, Mt, G, t1);     /* M^T G      */
                    mm(D, t1, Mt, carry);    /* M^T G M    */
                } else {
                    mm_nt(D, G, xp, t1);
                    memcpy(dM + o, t1, sizeof(double) * DD);
                    mm_tn(D, Mt, G, carry);
                }
            }
            if (dh0) memcpy(dh0 + (b * N + n) * DD, carry, sizeof(double) * DD);
        }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Cayley transform                                                          */
/* ------------------------------------------------------------------------ */
/* Q = (I - Om)^{-1} (I + Om)  (python/clifford_cl6.py:57-68,
 * python/clifford_cl8.py:29-45 with use_schulz=False) */
int orc_cayley(const double* Om, double* Q, long count, int D) {
    if (D < 1 || D > ORC_MAXD || count < 0) return 1;
    const long DD = (long)D * D;
    int bad = 0;
#pragma omp parallel for schedule(static) reduction(| : bad)
    for (long e = 0; e < count; ++e) {
        double A[ORC_MAXD * ORC_MAXD], Bm[ORC_MAXD * ORC_MAXD];
        for (int i = 0; i < D; ++i)
            for (int j = 0; j < D; ++j) {
                double id = (i == j) ? 1.0 : 0.0;
                A[i * D + j] = id - Om[e * DD + i * D + j];
                Bm[i * D + j] = id + Om[e * DD + i * D + j];
            }
        bad |= solve(D, A, Bm, Q + e * DD);
    }
    return bad;
}

/* ------------------------------------------------------------------------ */
/* fused rotor scan: generators + dt + gamma + S  ->  X                      */
/* ------------------------------------------------------------------------ */
/*
 * Per step (python/clifford_cl6.py:150-171, python/clifford_cl8.py:160-179):
 *   Om    = (sum_k g_k E_k) * (0.5 * dt)    E_k: skew basis [K, D, D]
 *   Q     = (I - Om)^{-1} (I + Om)
 *   damped (gamma != NULL):  a = sigmoid(-gamma * dt); M = sqrt(a) Q; C = (1 - a) S
 *   undamped (gamma == NULL): M = Q; C = S      (h_t = R h R~ + x_t)
 *   X = scan(M, C)
 * gens [B,T,N,K], dt [B,T], gamma [B,T,N], S [B,T,N,D,D].
 */
static void build_step(int D, int K, const double* basis, const double* g, double dt,
                       const double* gamma, const double* S, double* Om, double* Q,
                       double* M, double* Cc, double* alpha_out) {
    const int DD = D * D;
    for (int i = 0; i < DD; ++i) Om[i] = 0.0;
    for (int k = 0; k < K; ++k) {
        const double gk = g[k];
        if (gk == 0.0) continue;
        for (int i = 0; i < DD; ++i) Om[i] += gk * basis[k * DD + i];
    }
    for (int i = 0; i < DD; ++i) Om[i] *= 0.5 * dt;
    orc_cayley(Om, Q, 1, D);
    double a = 1.0;
    if (gamma) a = 1.0 / (1.0 + exp(gamma[0] * dt));
    const double sa = sqrt(a);
    for (int i = 0; i < DD; ++i) {
        M[i] = sa * Q[i];
        Cc[i] = gamma ? (1.0 - a) * S[i] : S[i];
    }
    *alpha_out = a;
}

int orc_rotor_build(const double* gens, const double* dt, const double* gamma, const double* S,
                    const double* basis, int K, double* M, double* C,
                    long B, long T, long N, int D) {
    if (D < 1 || D > ORC_MAXD || K < 0) return 1;
    const long DD = (long)D * D;
#pragma omp parallel for collapse(3) schedule(static)
    for (long b = 0; b < B; ++b)
        for (long t = 0; t < T; ++t)
            for (long n = 0; n < N; ++n) {
                double Om[ORC_MAXD * ORC_MAXD], Q[ORC_MAXD * ORC_MAXD], a;
                const size_t e = off3(b, t, n, T, N);
                build_step(D, K, basis, gens + e * K, dt[b * T + t], gamma ? gamma + e : NULL,
                           S + e * DD, Om, Q, M + e * DD, C + e * DD, &a);
            }
    return 0;
}

int orc_rotor_scan_fwd(const double* gens, const double* dt, const double* gamma, const double* S,
                       const double* basis, int K, const double* h0, double* X,
                       long B, long T, long N, int D, int two_sided) {
    if (D < 1 || D > ORC_MAXD || K < 0) return 1;
    const long DD = (long)D * D;
#pragma omp parallel for collapse(2) schedule(static)
    for (long b = 0; b < B; ++b)
        for (long n = 0; n < N; ++n) {
            double h[ORC_MAXD * ORC_MAXD], tmp[ORC_MAXD * ORC_MAXD];
            double Om[ORC_MAXD * ORC_MAXD], Q[ORC_MAXD * ORC_MAXD];
            double Mt[ORC_MAXD * ORC_MAXD], Ct[ORC_MAXD * ORC_MAXD], a;
            if (h0) memcpy(h, h0 + (b * N + n) * DD, sizeof(double) * DD);
            else memset(h, 0, sizeof(double) * DD);
            for (long t = 0; t < T; ++t) {
                const size_t e = off3(b, t, n, T, N);
                build_step(D, K, basis, gens + e * K, dt[b * T + t], gamma ? gamma + e : NULL,
                           S + e * DD, Om, Q, Mt, Ct, &a);
                mm(D, Mt, h, tmp);
                if (two_sided) mm_nt(D, tmp, Mt, tmp);
                for (long i = 0; i < DD; ++i) h[i] = tmp[i] + Ct[i];
                memcpy(X + e * DD, h, sizeof(double) * DD);
            }
        }
    return 0;
}

/*
 * Adjoint of orc_rotor_scan_fwd (what autograd computes through
 * python/clifford_cl6.py:150-171):
 *   scan adjoint gives dM_t, dC_t;
 *   dS = (1-a) dC;   da = -<dC, S> + <dM, Q> / (2 sqrt a)
 *   dQ = sqrt(a) dM; dOm = (I - Om)^{-T} dQ (I + Q)^T
 *   dg_k = <dOm, E_k> * 0.5 dt
 *   dt collects 0.5 * <dOm, sum_k g_k E_k> and da * a(1-a) * (-gamma), summed over n
 *   dgamma = da * a(1-a) * (-dt)
 * ddt is accumulated over channels; it is written, not added to.
 */
int orc_rotor_scan_bwd(const double* gens, const double* dt, const double* gamma, const double* S,
                       const double* basis, int K, const double* h0, const double* X,
                       const double* dX, double* dgens, double* ddt, double* dgamma, double* dS,
                       double* dh0, long B, long T, long N, int D, int two_sided) {
    if (D < 1 || D > ORC_MAXD || K < 0) return 1;
    const long DD = (long)D * D;
    double* ddt_part = (double*)calloc((size_t)(B * T * N > 0 ? B * T * N : 1), sizeof(double));
    if (!ddt_part) return 1;
#pragma omp parallel for collapse(2) schedule(static)
    for (long b = 0; b < B; ++b)
        for (long n = 0; n < N; ++n) {
            double carry[ORC_MAXD * ORC_MAXD], G[ORC_MAXD * ORC_MAXD], xp[ORC_MAXD * ORC_MAXD];
            double t1[ORC_MAXD * ORC_MAXD], t2[ORC_MAXD * ORC_MAXD], dMt[ORC_MAXD * ORC_MAXD];
            double Om[ORC_MAXD * ORC_MAXD], Q[ORC_MAXD * ORC_MAXD], Mt[ORC_MAXD * ORC_MAXD];
            double Ct[ORC_MAXD * ORC_MAXD], A[ORC_MAXD * ORC_MAXD], AT[ORC_MAXD * ORC_MAXD];
            double W[ORC_MAXD * ORC_MAXD], dOm[ORC_MAXD * ORC_MAXD], IQ[ORC_MAXD * ORC_MAXD];
            double a;
            memset(carry, 0, sizeof(double) * DD);
            for (long t = T - 1; t >= 0; --t) {
                const size_t e = off3(b, t, n, T, N);
                const double dtv = dt[b * T + t];
                build_step(D, K, basis, gens + e * K, dtv, gamma ? gamma + e : NULL, S + e * DD,
                           Om, Q, Mt, Ct, &a);
                for (long i = 0; i < DD; ++i) G[i] = dX[e * DD + i] + carry[i];
                if (t > 0) memcpy(xp, X + off3(b, t - 1, n, T, N) * DD, sizeof(double) * DD);
                else if (h0) memcpy(xp, h0 + (b * N + n) * DD, sizeof(double) * DD);
                else memset(xp, 0, sizeof(double) * DD);
                if (two_sided) {
                    mm(D, G, Mt, t1); mm_nt(D, t1, xp, t1);
                    mm(D, Mt, xp, t2); mm_tn(D, G, t2, t2);
                    for (long i = 0; i < DD; ++i) dMt[i] = t1[i] + t2[i];
                    mm_tn(D, Mt, G, t1); mm(D, t1, Mt, carry);
                } else {
                    mm_nt(D, G, xp, dMt);
                    mm_tn(D, Mt, G, carry);
                }
                /* dC = G */
                double da = 0.0;
                if (gamma) {
                    for (long i = 0; i < DD; ++i) dS[e * DD + i] = (1.0 - a) * G[i];
                    da = -dot(DD, G, S + e * DD) + dot(DD, dMt, Q) / (2.0 * sqrt(a));
                } else {
                    for (long i = 0; i < DD; ++i) dS[e * DD + i] = G[i];
                }
                const double sa = sqrt(a);
                for (long i = 0; i < DD; ++i) dMt[i] *= sa; /* dQ */
                /* dOm = A^{-T} dQ (I + Q)^T with A = I - Om: solve A^T W = dQ */
                for (int i = 0; i < D; ++i)
                    for (int j = 0; j < D; ++j) {
                        A[i * D + j] = ((i == j) ? 1.0 : 0.0) - Om[i * D + j];
                        IQ[i * D + j] = ((i == j) ? 1.0 : 0.0) + Q[i * D + j];
                    }
                for (int i = 0; i < D; ++i)
                    for (int j = 0; j < D; ++j) AT[i * D + j] = A[j * D + i];
                solve(D, AT, dMt, W);
                mm_nt(D, W, IQ, dOm);
                double ddt_acc = 0.0;
                for (int k = 0; k < K; ++k) {
                    const double proj = dot(DD, dOm, basis + k * DD);
                    dgens[e * K + k] = proj * 0.5 * dtv;
                    ddt_acc += proj * 0.5 * gens[e * K + k];
                }
                if (gamma) {
                    const double dz = da * a * (1.0 - a); /* d a / d z with z = -gamma dt */
                    dgamma[e] = -dz * dtv;
                    ddt_acc += -dz * gamma[e];
                }
                ddt_part[e] = ddt_acc;
            }
            if (dh0) memcpy(dh0 + (b * N + n) * DD, carry, sizeof(double) * DD);
        }
    for (long b = 0; b < B; ++b)
        for (long t = 0; t < T; ++t) {
            double s = 0.0;
            for (long n = 0; n < N; ++n) s += ddt_part[off3(b, t, n, T, N)];
            ddt[b * T + t] = s;
        }
    free(ddt_part);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* blade-basis geometric algebra Cl(p, 0)                                    */
/* ------------------------------------------------------------------------ */
/*
 * Basis blade i is orient[i] * e_{mask[i]} where e_m is the product of the basis
 * vectors in mask m taken in increasing index order.  Product of canonical
 * blades: e_a e_b = s(a, b) e_{a xor b}, s = (-1)^(number of pairs (i in a, j in b)
 * with j < i), all squares +1 (include/clifford_algebra.cuh:60-74).
 */
static int popc(unsigned x) { int c = 0; while (x) { c += x & 1u; x >>= 1; } return c; }
static double canon_sign(unsigned a, unsigned b) {
    int swaps = 0;
    for (int i = 0; i < 16; ++i)
        if (a & (1u << i))
            for (int j = 0; j < i; ++j)
                if (b & (1u << j)) ++swaps;
    return (swaps & 1) ? -1.0 : 1.0;
}

/* out[count, nbl] = a[count, nbl] * b[count, nbl] */
int orc_ga_product(const int* masks, const int* orient, int nbl, const double* a, const double* b,
                   double* out, long count) {
    if (nbl < 1 || nbl > 256) return 1;
    int* idx = (int*)malloc(sizeof(int) * 65536);
    if (!idx) return 1;
    for (int i = 0; i < 65536; ++i) idx[i] = -1;
    for (int i = 0; i < nbl; ++i) idx[masks[i]] = i;
    int bad = 0;
#pragma omp parallel for schedule(static) reduction(| : bad)
    for (long e = 0; e < count; ++e) {
        double acc[256];
        for (int i = 0; i < nbl; ++i) acc[i] = 0.0;
        for (int i = 0; i < nbl; ++i) {
            const double va = a[e * nbl + i];
            if (va == 0.0) continue;
            for (int j = 0; j < nbl; ++j) {
                const double vb = b[e * nbl + j];
                if (vb == 0.0) continue;
                const unsigned m = (unsigned)(masks[i] ^ masks[j]);
                const int k = idx[m];
                if (k < 0) { bad = 1; continue; }
                const double s = orient[i] * orient[j] * orient[k] * canon_sign(masks[i], masks[j]);
                acc[k] += s * va * vb;
            }
        }
        for (int i = 0; i < nbl; ++i) out[e * nbl + i] = acc[i];
    }
    free(idx);
    return bad;
}

/* reversion sign of a blade of grade g: (-1)^(g(g-1)/2) (include/clifford_algebra.cuh:127-138) */
static double rev_sign(int mask) { int g = popc((unsigned)mask); return ((g * (g - 1) / 2) & 1) ? -1.0 : 1.0; }

/* Cl(3,0) layout [1, e1, e2, e3, e12, e23, e31, e123] (include/clifford_configs.cuh:38-51). */
static const int G3_MASK[8] = {0, 1, 2, 4, 3, 6, 5, 7};
static const int G3_ORI[8] = {1, 1, 1, 1, 1, 1, -1, 1}; /* e31 = e3 e1 = -e1 e3 */
static double g3_tab_s[8][8];
static int g3_tab_k[8][8];
static int g3_ready = 0;
static void g3_init(void) {
    if (g3_ready) return;
    int idx[8];
    for (int i = 0; i < 8; ++i) idx[G3_MASK[i]] = i;
    for (int i = 0; i < 8; ++i)
        for (int j = 0; j < 8; ++j) {
            int k = idx[G3_MASK[i] ^ G3_MASK[j]];
            g3_tab_k[i][j] = k;
            g3_tab_s[i][j] = G3_ORI[i] * G3_ORI[j] * G3_ORI[k] * canon_sign(G3_MASK[i], G3_MASK[j]);
        }
    g3_ready = 1;
}
static void g3_mul(const double* a, const double* b, double* out) {
    double acc[8] = {0};
    for (int i = 0; i < 8; ++i)
        for (int j = 0; j < 8; ++j) acc[g3_tab_k[i][j]] += g3_tab_s[i][j] * a[i] * b[j];
    memcpy(out, acc, sizeof(acc));
}
static void g3_rev(const double* a, double* out) {
    for (int i = 0; i < 8; ++i) out[i] = rev_sign(G3_MASK[i]) * a[i];
}
/* rotor R = (1 - Om)^{-1} (1 + Om) for Om = 0.5 dt (g12 e12 + g23 e23 + g31 e31);
 * every Cl(3) bivector is simple, so R = (1 - w + 2 Om) / (1 + w), w = |Om|^2. */
static void g3_rotor(const double* g, double dt, double* R, double* Om3, double* w_out) {
    double om[3] = {0.5 * dt * g[0], 0.5 * dt * g[1], 0.5 * dt * g[2]};
    double w = om[0] * om[0] + om[1] * om[1] + om[2] * om[2];
    for (int i = 0; i < 8; ++i) R[i] = 0.0;
    R[0] = (1.0 - w) / (1.0 + w);
    R[4] = 2.0 * om[0] / (1.0 + w);
    R[5] = 2.0 * om[1] / (1.0 + w);
    R[6] = 2.0 * om[2] / (1.0 + w);
    if (Om3) { Om3[0] = om[0]; Om3[1] = om[1]; Om3[2] = om[2]; }
    if (w_out) *w_out = w;
}

/*
 * Cl(3,0) affine rotor scan in the blade basis: h_t = R_t h_{t-1} R~_t + x_t with
 * h_{-1} = h0 (zero when NULL).  gens [B,T,N,3] on (e12, e23, e31), dt [B,T],
 * x, h [B,T,N,8].
 */
int orc_ga3_scan_fwd(const double* gens, const double* dt, const double* x, const double* h0,
                     double* h, long B, long T, long N) {
    g3_init();
#pragma omp parallel for collapse(2) schedule(static)
    for (long b = 0; b < B; ++b)
        for (long n = 0; n < N; ++n) {
            double st[8], R[8], Rr[8], t1[8];
            if (h0) memcpy(st, h0 + (b * N + n) * 8, sizeof(st));
            else memset(st, 0, sizeof(st));
            for (long t = 0; t < T; ++t) {
                const size_t e = off3(b, t, n, T, N);
                g3_rotor(gens + e * 3, dt[b * T + t], R, NULL, NULL);
                g3_rev(R, Rr);
                g3_mul(R, st, t1);
                g3_mul(t1, Rr, st);
                for (int i = 0; i < 8; ++i) st[i] += x[e * 8 + i];
                memcpy(h + e * 8, st, sizeof(st));
            }
        }
    return 0;
}

/*
 * Adjoint of orc_ga3_scan_fwd.  With L_t(v) = R_t v R~_t:
 *   g_t = dh_t + L_{t+1}^T(g_{t+1}); dx_t = g_t;
 *   dR_m = <g_t, E_m h_{t-1} R~ + R h_{t-1} E~_m> for the even basis E_m;
 *   dOm from R(Om) = (1 - w + 2 Om)/(1 + w); dgens = 0.5 dt dOm;
 *   ddt[b,t] = sum_n 0.5 <dOm, g>.
 */
int orc_ga3_scan_bwd(const double* gens, const double* dt, const double* h0, const double* h,
                     const double* dh, double* dgens, double* ddt, double* dx, double* dh0,
                     long B, long T, long N) {
    g3_init();
    double* part = (double*)calloc((size_t)(B * T * N > 0 ? B * T * N : 1), sizeof(double));
    if (!part) return 1;
    static const int EVEN[4] = {0, 4, 5, 6};
#pragma omp parallel for collapse(2) schedule(static)
    for (long b = 0; b < B; ++b)
        for (long n = 0; n < N; ++n) {
            double carry[8] = {0}, g[8], hp[8], R[8], Rr[8], om[3], w;
            for (long t = T - 1; t >= 0; --t) {
                const size_t e = off3(b, t, n, T, N);
                const double dtv = dt[b * T + t];
                for (int i = 0; i < 8; ++i) g[i] = dh[e * 8 + i] + carry[i];
                memcpy(dx + e * 8, g, sizeof(g));
                if (t > 0) memcpy(hp, h + off3(b, t - 1, n, T, N) * 8, sizeof(hp));
                else if (h0) memcpy(hp, h0 + (b * N + n) * 8, sizeof(hp));
                else memset(hp, 0, sizeof(hp));
                g3_rotor(gens + e * 3, dtv, R, om, &w);
                g3_rev(R, Rr);
                /* dR over the even basis */
                double dR[4];
                for (int m = 0; m < 4; ++m) {
                    double Em[8] = {0}, Emr[8], a1[8], a2[8];
                    Em[EVEN[m]] = 1.0;
                    g3_rev(Em, Emr);
                    g3_mul(Em, hp, a1); g3_mul(a1, Rr, a1);
                    g3_mul(R, hp, a2); g3_mul(a2, Emr, a2);
                    double s = 0.0;
                    for (int i = 0; i < 8; ++i) s += g[i] * (a1[i] + a2[i]);
                    dR[m] = s;
                }
                /* R0 = (1-w)/(1+w), Rb = 2 om_b/(1+w) */
                const double den = 1.0 + w, den2 = den * den;
                double dom[3];
                for (int bb = 0; bb < 3; ++bb) {
                    double v = dR[0] * (-4.0 * om[bb] / den2);
                    for (int c = 0; c < 3; ++c)
                        v += dR[1 + c] * (((bb == c) ? 2.0 / den : 0.0) - 4.0 * om[c] * om[bb] / den2);
                    dom[bb] = v;
                }
                double acc = 0.0;
                for (int bb = 0; bb < 3; ++bb) {
                    dgens[e * 3 + bb] = 0.5 * dtv * dom[bb];
                    acc += 0.5 * gens[e * 3 + bb] * dom[bb];
                }
                part[e] = acc;
                /* carry = L_t^T(g) = R~ g R (L_t is orthogonal for a unit rotor) */
                {
                    double a1[8];
                    g3_mul(Rr, g, a1);
                    g3_mul(a1, R, carry);
                }
            }
            if (dh0) memcpy(dh0 + (b * N + n) * 8, carry, sizeof(carry));
        }
    for (long b = 0; b < B; ++b)
        for (long t = 0; t < T; ++t) {
            double s = 0.0;
            for (long n = 0; n < N; ++n) s += part[off3(b, t, n, T, N)];
            ddt[b * T + t] = s;
        }
    free(part);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Clifford-LTC cell (python/clifford_layer.py:50-115)                       */
/* ------------------------------------------------------------------------ */
/*
 * One recurrent step, 4 x 4 matrix form:
 *   S_i   = sum_j W_rec[i,j] X_j + sum_k W_in[i,k] x_k
 *   gamma = softplus(gamma_bias_i + 0.25 tr S_i)
 *   Om    = 0.5 (S - S^T) * 0.5 dt
 *   Q     = (I + Om)(I - Om) / (1 + 0.25 * 0.5 |Om|_F^2)
 *   next  = sig(-gamma dt) Q X_i Q^T + (1 - sig(-gamma dt)) S_i
 * prev [Bt,N,16], x [Bt,in_dim], W_rec [N,N,16], W_in [N,in_dim,16], gamma_bias [N].
 */
static double softplus(double v) { return v > 20.0 ? v : log1p(exp(v)); }
static double sigm(double v) { return 1.0 / (1.0 + exp(-v)); }

int orc_cell_fwd(const double* prev, const double* x, const double* W_rec, const double* W_in,
                 const double* gamma_bias, double dt, double* out, long Bt, long N, long in_dim) {
#pragma omp parallel for collapse(2) schedule(static)
    for (long b = 0; b < Bt; ++b)
        for (long i = 0; i < N; ++i) {
            double S[16] = {0}, Om[16], P[16], Mn[16], Q[16], t1[16];
            for (long j = 0; j < N; ++j) {
                mm(4, W_rec + (i * N + j) * 16, prev + (b * N + j) * 16, t1);
                for (int c = 0; c < 16; ++c) S[c] += t1[c];
            }
            for (long k = 0; k < in_dim; ++k)
                for (int c = 0; c < 16; ++c) S[c] += W_in[(i * in_dim + k) * 16 + c] * x[b * in_dim + k];
            const double tr = S[0] + S[5] + S[10] + S[15];
            const double gam = softplus(gamma_bias[i] + 0.25 * tr);
            double nrm = 0.0;
            for (int r = 0; r < 4; ++r)
                for (int c = 0; c < 4; ++c) {
                    Om[r * 4 + c] = 0.5 * (S[r * 4 + c] - S[c * 4 + r]) * (0.5 * dt);
                    nrm += Om[r * 4 + c] * Om[r * 4 + c];
                }
            const double den = 1.0 + 0.25 * (0.5 * nrm);
            for (int r = 0; r < 4; ++r)
                for (int c = 0; c < 4; ++c) {
                    P[r * 4 + c] = ((r == c) ? 1.0 : 0.0) + Om[r * 4 + c];
                    Mn[r * 4 + c] = ((r == c) ? 1.0 : 0.0) - Om[r * 4 + c];
                }
            mm(4, P, Mn, Q);
            for (int c = 0; c < 16; ++c) Q[c] /= den;
            mm(4, Q, prev + (b * N + i) * 16, t1);
            mm_nt(4, t1, Q, t1);
            const double dec = sigm(-gam * dt);
            for (int c = 0; c < 16; ++c) out[(b * N + i) * 16 + c] = dec * t1[c] + (1.0 - dec) * S[c];
        }
    return 0;
}
