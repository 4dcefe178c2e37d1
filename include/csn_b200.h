/*
 * csn_b200.h -- C ABI of the B200 (sm_100a) rotor-scan library libcsn_b200.so.
 *
 * Plain C: raw device pointers, sizes and a cudaStream_t passed as void*.  No torch
 * types cross this boundary.  Every entry point returns a status code (CSN_OK = 0)
 * and records a message retrievable with csn_last_error() on the calling thread.
 * Launches are asynchronous on `stream` (NULL = legacy default stream); a status of
 * CSN_OK means the launches were queued, not that they finished.
 *
 * Tensor layout is the reference's: float32, row-major, contiguous,
 *   M, C, S, X, dX, dM, dC, dS : [B, T, N, D, D]     element (b,t,n) at ((b*T+t)*N+n)*D*D
 *   gens, dgens                : [B, T, N, K]        K = D(D-1)/2 (basis TRIU) or the
 *                                                    GA bivector count (basis GA)
 *   dt, ddt                    : [B, T]              one time step per token, shared by channels
 *   gamma, dgamma              : [B, T, N]           post-softplus decay rate
 *   h0, dh0                    : [B, N, D, D]        optional initial state (NULL = zero)
 * Device pointers must be 16-byte aligned (8-byte for gens/dgens when K % 4 != 0).
 *
 * Workspace: entry points that take (workspace, workspace_bytes) use scratch device
 * memory of at least the size the matching *_workspace_bytes() query returns.  Pass
 * workspace = NULL to let the library allocate it stream-ordered (cudaMallocAsync /
 * cudaFreeAsync on `stream`).
 *
 * Each declaration names the reference interface it replaces (paths relative to the
 * reference project root).
 */
#ifndef CSN_B200_H
#define CSN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum csn_status {
  CSN_OK = 0,
  CSN_ERR_INVALID = 1,     /* bad shape, pointer, alignment or size */
  CSN_ERR_UNSUPPORTED = 2, /* a D / basis / mode this build does not provide */
  CSN_ERR_CUDA = 3,        /* a CUDA runtime call or launch failed */
  CSN_ERR_TIMEOUT = 4      /* a bounded device-side wait gave up */
};

enum csn_basis {
  CSN_BASIS_TRIU = 0, /* g_k at torch.triu_indices(D, D, 1)[:, k] (python/clifford_cl6.py:124-125) */
  CSN_BASIS_GA = 1    /* GA bivector blades e_ij (i<j, lexicographic) mapped through a real
                         representation: Cl(3,0) on R^4 (D = 4), Cl(8,0) on R^16 (D = 16) */
};

/* Library version string and the message of the last failing call on this thread. */
const char* csn_version(void);
const char* csn_last_error(void);

/* ------------------------------------------------------------------ plain scan */
size_t csn_scan_workspace_bytes(int64_t B, int64_t T, int64_t N, int D);

/* Plain-scan flags: bit 0 two-sided (X_t = M_t X_{t-1} M_t^T + C_t, else M_t X_{t-1} + C_t),
 * bit 1 reverse time (the scan runs from t = T-1 down to 0: X_t = M_t X_{t+1} (M_t^T) + C_t,
 * X_T = h0 or 0) -- the flipped scan of the reference's bidirectional spatial scan
 * (csn_toolkit/csn/vision.py:97-107) without flipping any tensor.  flags = 0 / 1 are the
 * former one-sided / two-sided values. */
#define CSN_SCAN_TWO_SIDED 1
#define CSN_SCAN_REVERSE 2

/* X_t = M_t X_{t-1} M_t^T + C_t (two-sided) or M_t X_{t-1} + C_t, X_{-1} = h0 or 0.
 * Replaces python/clifford_scan.py:41 parallel_rotor_scan (two-sided default),
 * csn_toolkit/csn/scan.py:24 CliffordScanFunction.forward, and the pybind entry
 * scan_fwd_cuda_d4(M, C) -> X of csn_toolkit/csn/cuda/scan_cuda.cpp:6 ([S,T,4,4] is
 * B = S, N = 1, D = 4, flags = 0).  D in {4, 8, 16}. */
int csn_scan_fwd(const float* M, const float* C, const float* h0, float* X,
                 int64_t B, int64_t T, int64_t N, int D, int flags,
                 void* workspace, size_t workspace_bytes, void* stream);

/* Reverse-time adjoint of csn_scan_fwd: dM, dC (and dh0 when h0 and dh0 are given).
 * Replaces csn_toolkit/csn/scan.py:44 CliffordScanFunction.backward, autograd through
 * python/clifford_scan.py:41, and scan_bwd_cuda_d4(M, X, grad_X) -> [grad_M, grad_C]
 * of csn_toolkit/csn/cuda/scan_cuda.cpp:7.  dM of the first scanned step is 0 when h0 is
 * NULL, as in the reference.  Same flags as csn_scan_fwd. */
int csn_scan_bwd(const float* M, const float* X, const float* dX, const float* h0,
                 float* dM, float* dC, float* dh0,
                 int64_t B, int64_t T, int64_t N, int D, int flags,
                 void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------ fused rotor scan */
size_t csn_rotor_scan_workspace_bytes(int64_t B, int64_t T, int64_t N, int D);

/* Generators + dt + gamma + S -> X in one pass, never materialising M or C:
 *   Omega = 0.5 dt sum_k g_k E_k,  Q = (I - Omega)^{-1} (I + Omega),
 *   gamma != NULL: a = sigmoid(-gamma dt), M = sqrt(a) Q, C = (1 - a) S
 *   gamma == NULL: M = Q, C = S     (h_t = R_t h_{t-1} R~_t + x_t)
 *   X = scan(M, C).
 * Replaces the scan section of CliffordCL6Block.forward (python/clifford_cl6.py:150-171)
 * and CliffordCL8Block.forward (python/clifford_cl8.py:160-179): cayley_rotor_8x8 /
 * cayley_rotor_16x16 + parallel_rotor_scan. */
int csn_rotor_scan_fwd(const float* gens, const float* dt, const float* gamma, const float* S,
                       const float* h0, float* X,
                       int64_t B, int64_t T, int64_t N, int D, int basis, int two_sided,
                       void* workspace, size_t workspace_bytes, void* stream);

/* Adjoint of csn_rotor_scan_fwd (what autograd computes through the same reference
 * lines): dgens, ddt [B,T] (summed over channels), dgamma (damped only), dS, dh0. */
int csn_rotor_scan_bwd(const float* gens, const float* dt, const float* gamma, const float* S,
                       const float* h0, const float* X, const float* dX,
                       float* dgens, float* ddt, float* dgamma, float* dS, float* dh0,
                       int64_t B, int64_t T, int64_t N, int D, int basis, int two_sided,
                       void* workspace, size_t workspace_bytes, void* stream);

/* csn_rotor_scan_bwd for a backward that follows its forward on the same workspace: the
 * workspace must be the one given to csn_rotor_scan_fwd with the same gens, dt, gamma, B, T,
 * N, D and basis, unused since; the chunk rotor products that forward left in it are reused,
 * so the backward's reduce pass skips them.  Same results as csn_rotor_scan_bwd to fp32
 * rounding.  Replaces the same reference code (autograd keeps the forward's intermediates). */
int csn_rotor_scan_bwd_reuse(const float* gens, const float* dt, const float* gamma, const float* S,
                             const float* h0, const float* X, const float* dX,
                             float* dgens, float* ddt, float* dgamma, float* dS, float* dh0,
                             int64_t B, int64_t T, int64_t N, int D, int basis, int two_sided,
                             void* workspace, size_t workspace_bytes, void* stream);

/* Rotor cache for D = 16 (where building a rotor costs as much as the scan step itself):
 *   csn_rotor_scan_fwd_cached: csn_rotor_scan_fwd that also stores every step's matrix
 *                              M_t = sqrt(a_t) Q_t in Mcache ([B,T,N,16,16], the layout of S);
 *                              its apply pass reuses what its reduce pass stored;
 *   csn_rotor_scan_bwd_cached: csn_rotor_scan_bwd that loads M_t from that Mcache instead
 *                              of rebuilding the Cayley rotors (same other inputs as the forward).
 * Same results as the uncached pair to fp32 rounding.  D != 16 -> CSN_ERR_UNSUPPORTED.  Replaces
 * the same reference code as csn_rotor_scan_fwd/bwd (python/clifford_cl8.py:160-179, where
 * autograd keeps the rotors Q between forward and backward). */
int csn_rotor_scan_fwd_cached(const float* gens, const float* dt, const float* gamma,
                              const float* S, const float* h0, float* X, float* Mcache,
                              int64_t B, int64_t T, int64_t N, int D, int basis, int two_sided,
                              void* workspace, size_t workspace_bytes, void* stream);
int csn_rotor_scan_bwd_cached(const float* gens, const float* dt, const float* gamma,
                              const float* S, const float* h0, const float* X, const float* dX,
                              const float* Mcache, float* dgens, float* ddt, float* dgamma,
                              float* dS, float* dh0, int64_t B, int64_t T, int64_t N, int D,
                              int basis, int two_sided, void* workspace, size_t workspace_bytes,
                              void* stream);

/* Multi-head layout with one dt per head (python/clifford_multihead.py:137-170): the
 * N = H * Nh channels are H heads of Nh neurons and
 *   gens [B,T,H,Nh,K], dt [B,T,H], gamma [B,T,H,Nh] (NULL = undamped), S, X, dX, dS
 *   [B,T,H,Nh,D,D], h0, dh0 [B,H,Nh,D,D], ddt [B,T,H];
 * neuron (h, i) uses dt[b,t,h].  The recurrence of every neuron is the one of
 * csn_rotor_scan_fwd/bwd; the reference gets the same numbers by folding heads into the batch
 * ([B*H, T, Nh], python/clifford_multihead.py:157-163) with transposed copies of Omega, S and
 * the decay, which these entry points read in place instead.  ddt is summed over each head's
 * neurons.  Workspace: csn_rotor_scan_workspace_bytes(B, T, H * Nh, D).
 *   Mcache: NULL, or (D = 16 only, as csn_rotor_scan_fwd_cached / _bwd_cached) the step
 *           rotors [B,T,H,Nh,16,16] that the forward stores and the backward loads;
 *   reuse:  1 = the workspace is the one the forward used (as csn_rotor_scan_bwd_reuse). */
int csn_rotor_scan_heads_fwd(const float* gens, const float* dt, const float* gamma,
                             const float* S, const float* h0, float* X, float* Mcache,
                             int64_t B, int64_t T, int64_t H, int64_t Nh, int D, int basis,
                             int two_sided, void* workspace, size_t workspace_bytes, void* stream);
int csn_rotor_scan_heads_bwd(const float* gens, const float* dt, const float* gamma,
                             const float* S, const float* h0, const float* X, const float* dX,
                             const float* Mcache, float* dgens, float* ddt, float* dgamma,
                             float* dS, float* dh0, int64_t B, int64_t T, int64_t H, int64_t Nh,
                             int D, int basis, int two_sided, int reuse, void* workspace,
                             size_t workspace_bytes, void* stream);

/* Same computation and chunking as csn_rotor_scan_fwd (bit-identical results), for
 * callers that cannot allocate device memory: hosts that hand the whole GPU to their
 * own memory pool, or loops that must not allocate once running.  No counterpart in
 * the reference (whose extension allocates every output with torch::empty_like,
 * csn_toolkit/csn/cuda/scan_cuda.cu:237).  The caller still passes every input and X.
 * Scratch comes from a static 32 MiB device array that the library holds on every GPU
 * that loads it, until process exit; problems whose csn_scan_workspace_bytes(B, T, N, D)
 * exceeds 33554432 bytes are rejected with CSN_ERR_INVALID.  The first call on a device
 * looks up that array's device address (cudaGetSymbolAddress), so make it before any
 * stream capture.  The address is cached per device ordinal for the life of the process:
 * after cudaDeviceReset (or anything else that destroys the device's primary context and
 * so reloads the module) the cached address is stale, and the entry point must not be
 * called again on that device.  All calls share the one array: calls that overlap on the GPU (other
 * streams, other threads) race and must be serialised by the caller.  No scratch word
 * needs to start at zero: every word a call reads is written earlier in that call. */
int csn_rotor_scan_fwd_noalloc(const float* gens, const float* dt, const float* gamma,
                               const float* S, const float* h0, float* X,
                               int64_t B, int64_t T, int64_t N, int D, int basis, int two_sided,
                               void* stream);

/* ------------------------------------------------ sequence-parallel shard aggregates */
/* Summaries of one time shard (the local [B, T, N, ...] slice of a longer sequence) for the
 * cross-GPU carry exchange of the sequence-parallel scan.  The reference has no distributed
 * code; these are the chunk aggregates of its associative operator (python/clifford_scan.py:19-38)
 * taken over a whole shard:
 *   csn_rotor_scan_aggregate:     P_out = M_{T-1} ... M_0, c_out = final state of the shard's
 *                                 scan from zero (both [B, N, D, D]);
 *   csn_rotor_scan_bwd_aggregate: c_out = gradient leaving the shard at its first step when
 *                                 no gradient enters from its right end. */
size_t csn_rotor_scan_aggregate_workspace_bytes(int64_t B, int64_t T, int64_t N, int D);
int csn_rotor_scan_aggregate(const float* gens, const float* dt, const float* gamma, const float* S,
                             float* P_out, float* c_out, int64_t B, int64_t T, int64_t N, int D,
                             int basis, int two_sided, void* workspace, size_t workspace_bytes,
                             void* stream);
int csn_rotor_scan_bwd_aggregate(const float* gens, const float* dt, const float* gamma,
                                 const float* dX, float* c_out, int64_t B, int64_t T, int64_t N,
                                 int D, int basis, int two_sided, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* Resume the shard after its aggregate: the aggregate calls leave every chunk's aggregate in
 * `workspace`, and these calls (same inputs, same workspace, later on the same stream) run only
 * the carry and apply passes from them, so a shard's inputs are reduced once per direction.
 *   csn_rotor_scan_fwd_resume: csn_rotor_scan_fwd with carry-in h0 (NULL = zero);
 *   csn_rotor_scan_bwd_resume: csn_rotor_scan_bwd with dh_right [B,N,D,D] (NULL = zero), the
 *                              gradient entering after the shard's last step.
 * The workspace is required (>= csn_rotor_scan_aggregate_workspace_bytes).  The reference has
 * no sequence-parallel scan; these follow the scan of python/clifford_cl6.py:150-171. */
int csn_rotor_scan_fwd_resume(const float* gens, const float* dt, const float* gamma,
                              const float* S, const float* h0, float* X, int64_t B, int64_t T,
                              int64_t N, int D, int basis, int two_sided, void* workspace,
                              size_t workspace_bytes, void* stream);
int csn_rotor_scan_bwd_resume(const float* gens, const float* dt, const float* gamma,
                              const float* S, const float* h0, const float* X, const float* dX,
                              const float* dh_right, float* dgens, float* ddt, float* dgamma,
                              float* dS, float* dh0, int64_t B, int64_t T, int64_t N, int D,
                              int basis, int two_sided, void* workspace, size_t workspace_bytes,
                              void* stream);

/* O(1)-state generation step, in place: h <- M h M^T + C (one-sided: M h + C) with M, C built
 * from this step's gens [B,N,K], dt [B], gamma [B,N] (NULL = undamped) and S [B,N,D,D];
 * h [B,N,D,D].  Allocates nothing and launches one kernel, so a decode loop can capture it
 * in a CUDA graph.  The reference has no step API: its generation re-runs the whole model
 * on the growing prefix (tests/profile_performance.py:58-66); this is the recurrence of
 * python/clifford_cl6.py:150-171 advanced by one token. */
int csn_rotor_step(const float* gens, const float* dt, const float* gamma, const float* S, float* h,
                   int64_t B, int64_t N, int D, int basis, int two_sided, void* stream);

/* csn_rotor_step for a chain of steps on one stream (a captured decode loop), same arguments
 * and result.  For D = 8, triu basis, the kernel is launched with programmatic stream
 * serialization: it builds its rotor while the kernel before it on the stream is still running
 * and reads h only after that kernel has completed.  Contract: gens, dt, gamma and S of the
 * step must not be written by the kernel launched just before it on the stream (they are in
 * place before the chain starts); h may be.  Other D and bases launch as csn_rotor_step. */
int csn_rotor_step_chained(const float* gens, const float* dt, const float* gamma, const float* S,
                           float* h, int64_t B, int64_t N, int D, int basis, int two_sided,
                           void* stream);

/* -------------------------------------------------------------------- Cayley */
/* Q = (I - Omega)^{-1} (I + Omega) for `count` skew D x D matrices.
 * Replaces cayley_rotor_8x8 (python/clifford_cl6.py:57) and cayley_rotor_16x16 /
 * cayley_rotor_4x4 with use_schulz=False (python/clifford_cl8.py:29,65). */
int csn_cayley_fwd(const float* Omega, float* Q, int64_t count, int D, void* stream);

/* dOmega = (I - Omega)^{-T} dQ (I + Q)^T = 0.5 (I + Q)^T dQ (I + Q)^T (needs only Q):
 * the autograd of torch.linalg.solve in the same reference functions. */
int csn_cayley_bwd(const float* Q, const float* dQ, float* dOmega, int64_t count, int D,
                   void* stream);

/* ---------------------------------------------------- Cl(3,0) blade-basis scan */
/* h_t = R_t h_{t-1} R~_t + x_t with R_t = (1 - Om)^{-1}(1 + Om), Om = dt/2 (g12 e12 + g23 e23 +
 * g31 e31), h_{-1} = h0 or 0.  Multivectors [B,T,N,8] in the layout [1,e1,e2,e3,e12,e23,e31,e123]
 * of include/clifford_configs.cuh:38-51; gens [B,T,N,3]; dt [B,T].  The reference has no
 * Cl(3) scan: this is the blade-basis form of python/clifford_scan.py:41 (two-sided) with
 * the generated product tables of include/clifford_algebra.cuh:60-74. */
size_t csn_ga3_workspace_bytes(int64_t B, int64_t T, int64_t N);
int csn_ga3_scan_fwd(const float* gens, const float* dt, const float* x, const float* h0, float* h,
                     int64_t B, int64_t T, int64_t N, void* workspace, size_t workspace_bytes,
                     void* stream);
/* Adjoint: dx, dgens, ddt [B,T] (summed over channels), dh0 (when h0 and dh0 are given). */
int csn_ga3_scan_bwd(const float* gens, const float* dt, const float* h0, const float* h,
                     const float* dh, float* dgens, float* ddt, float* dx, float* dh0, int64_t B,
                     int64_t T, int64_t N, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------- Clifford cell */
/* One step of the Clifford-LTC cell, python/clifford_layer.py:50-115 (CliffordTENNCell.
 * forward, 4 x 4 matrix form with the symmetric rational rotor of that file):
 *   S_i = sum_j W_rec[i,j] X_j + sum_k W_in[i,k] x_k;  gamma = softplus(gamma_bias_i + tr S_i / 4)
 *   Om = (S - S^T) dt / 4;  Q = (I + Om)(I - Om) / (1 + |Om|_F^2 / 8)
 *   next = sig(-gamma dt) Q X_i Q^T + (1 - sig(-gamma dt)) S_i
 * prev/next [Bt, N, 16], x [Bt, in_dim], W_rec [N, N, 16], W_in [N, in_dim, 16], gamma_bias [N].
 * Replaces launch_clifford_cfc_forward (include/clifford_tenn_cell.cuh:50-55) with the
 * semantics of the Python module, which is the one the reference's models call. */
int csn_cell_fwd(const float* prev, const float* x, const float* W_rec, const float* W_in,
                 const float* gamma_bias, float dt, float* next, int64_t Bt, int64_t N,
                 int64_t in_dim, void* stream);

size_t csn_cell_workspace_bytes(int64_t Bt, int64_t N);

/* Exact adjoint of csn_cell_fwd (what autograd computes through the same lines): dprev,
 * dx, dW_rec, dW_in, dgamma_bias.  Outputs are written, not accumulated (the reference's
 * launch_clifford_cfc_backward, include/clifford_tenn_cell.cuh:57-63, accumulates with
 * atomics into caller-zeroed buffers).  dx, dW_rec, dW_in, dgamma_bias may be NULL. */
int csn_cell_bwd(const float* prev, const float* x, const float* W_rec, const float* W_in,
                 const float* gamma_bias, float dt, const float* dnext, float* dprev, float* dx,
                 float* dW_rec, float* dW_in, float* dgamma_bias, int64_t Bt, int64_t N,
                 int64_t in_dim, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------- block kernels around the scan */
/* Event spike of the scan output (python/clifford_scan.py:90-116 surrogate_spike on the
 * Frobenius energy, python/clifford_cl6.py:174-176, clifford_cl8.py:184-186,
 * clifford_multihead.py:176-178, clifford_model.py:190-192): for each of the n D x D states,
 *   Xs = X * [||X||_F - threshold >= 0]
 * and the surrogate adjoint (fast sigmoid 1 / (1 + beta |e - threshold|)^2 on the energy e):
 *   dX = [e >= threshold] dXs + (<dXs, X> / (1 + beta |e - threshold|)^2 / e) X   (0 at e = 0).
 * D in {4, 8, 16}; pointers 16-byte aligned. */
int csn_spike_fwd(const float* X, float* Xs, int64_t n, int D, float threshold, void* stream);
int csn_spike_bwd(const float* X, const float* dXs, float* dX, int64_t n, int D, float threshold,
                  float beta, void* stream);

/* LayerNorm over rows of C features (nn.LayerNorm(C, eps) of the blocks' ln_1 / ln_2 and the
 * LM's ln_f, python/clifford_cl6.py:94,121,229 applied at :140,184,272): y = (x - mean) * rstd * weight + bias,
 * rstd = 1 / sqrt(biased var + eps); mean and rstd [R] are kept for the backward.
 * 0 < C <= 1024, C % 4 == 0 (CSN_ERR_UNSUPPORTED otherwise); x, y, dy, dx, weight 16-byte
 * aligned.  The backward writes dx [R, C] and, when given, dweight and dbias [C]; its
 * workspace holds per-CTA partial sums (csn_layer_norm_bwd_workspace_bytes). */
int csn_layer_norm_fwd(const float* x, const float* weight, const float* bias, float* y, float* mean,
                       float* rstd, int64_t R, int C, float eps, void* stream);
size_t csn_layer_norm_bwd_workspace_bytes(int64_t R, int C);
int csn_layer_norm_bwd(const float* dy, const float* x, const float* mean, const float* rstd,
                       const float* weight, float* dx, float* dweight, float* dbias, int64_t R, int C,
                       void* workspace, size_t workspace_bytes, void* stream);

/* The blocks' input chain ln_1 -> causal depthwise conv1d -> SiLU (python/clifford_cl6.py:140-142,
 * clifford_cl8.py, clifford_multihead.py, clifford_model.py: nn.LayerNorm(C), then
 * nn.Conv1d(C, C, K, padding=K-1, groups=C) on the transposed sequence keeping the first T
 * outputs, then F.silu), fused:
 *   y[b,t,c] = silu(conv_bias[c] + sum_{j<K} conv_weight[c,0,j] * ln(x)[b, t-K+1+j, c])
 * with ln rows before t = 0 taken as 0.  x, y [B, T, C]; conv_weight [C, 1, K]; mean, rstd
 * [B*T] are the LayerNorm statistics the backward reuses.  The backward writes dx and, when
 * given, the four parameter gradients (its workspace holds per-CTA partial sums).
 * 0 < C <= 256, C % 4 == 0, 1 <= K <= 4 (CSN_ERR_UNSUPPORTED otherwise); x, y, dy, dx,
 * ln_weight, ln_bias, conv_bias 16-byte aligned. */
int csn_ln_conv_silu_fwd(const float* x, const float* ln_weight, const float* ln_bias,
                         const float* conv_weight, const float* conv_bias, float* y, float* mean,
                         float* rstd, int64_t B, int64_t T, int C, int K, float eps, void* stream);
size_t csn_ln_conv_silu_bwd_workspace_bytes(int64_t B, int64_t T, int C, int K);
int csn_ln_conv_silu_bwd(const float* dy, const float* x, const float* mean, const float* rstd,
                         const float* ln_weight, const float* ln_bias, const float* conv_weight,
                         const float* conv_bias, float* dx, float* dln_weight, float* dln_bias,
                         float* dconv_weight, float* dconv_bias, int64_t B, int64_t T, int C, int K,
                         void* workspace, size_t workspace_bytes, void* stream);

/* Least-action regulariser of the LMs (python/clifford_cl6.py:257-262, the same lines of
 * clifford_cl8.py and clifford_multihead.py) on the generator coefficients instead of Omega:
 * rows (b, t) of R = N * K coefficients biv [B, T, R] in H heads of R / H, dt [B, T, H];
 * w = 0.5 dt biv;  out[0] = c_kin * sum w^2,  out[1] = c_smooth * sum_{t >= 1} (w_t - w_{t-1})^2
 * (device scalars; the sums are reduced in a fixed order).  With c_kin = 2K / (D^2 * B*T*R) and
 * c_smooth = 2K / (D^2 * B*(T-1)*R) these are (Omega^2).mean() and
 * ((Omega[:, 1:] - Omega[:, :-1])^2).mean() of Omega = skew(biv) * 0.5 dt (D x D, K generators).
 * The backward takes dL/dout[0], dL/dout[1] as device pointers (NULL = 0) and writes dbiv
 * [B, T, R] and ddt [B, T, H] (either may be NULL). */
size_t csn_generator_action_workspace_bytes(int64_t B, int64_t T);
int csn_generator_action_fwd(const float* biv, const float* dt, int64_t B, int64_t T, int R, int H,
                             float c_kin, float c_smooth, float* out, void* workspace,
                             size_t workspace_bytes, void* stream);
int csn_generator_action_bwd(const float* biv, const float* dt, const float* g_kin,
                             const float* g_smooth, int64_t B, int64_t T, int R, int H, float c_kin,
                             float c_smooth, float* dbiv, float* ddt, void* stream);

/* Projection epilogue of the blocks (python/clifford_cl6.py:144-155; clifford_cl8.py,
 * clifford_multihead.py likewise): the generator, decay and time projections computed as one
 * GEMM give raw [R, Q] with Q = N*K + N + HT columns [generators | gamma | time]; the forward
 * writes the scan's inputs
 *   biv[r, n, k] = raw[r, n*K + k] * omega_scale[n],   gamma[r, n] = softplus(raw[r, N*K + n]),
 *   dt[r, h] = softplus(raw[r, N*K + N + h]) * dt_base          (softplus(x) = x for x > 20);
 * the backward writes draw [R, Q] from dbiv, dgamma, ddt (each may be NULL = 0) and
 * scale_part[r, n] = sum_k dbiv[r, n, k] raw[r, n*K + k], whose column sum is d omega_scale. */
int csn_projection_epilogue_fwd(const float* raw, int64_t R, int N, int K, int HT,
                                const float* omega_scale, float dt_base, float* biv, float* gamma,
                                float* dt, void* stream);
int csn_projection_epilogue_bwd(const float* raw, int64_t R, int N, int K, int HT,
                                const float* omega_scale, float dt_base, const float* dbiv,
                                const float* dgamma, const float* ddt, float* draw,
                                float* scale_part, void* stream);

/* out[c] = sum_r x[r, c] for x [R, C] row-major, summed in a fixed order (deterministic): the
 * bias gradients of the blocks' projections.  Workspace: csn_column_sum_workspace_bytes. */
size_t csn_column_sum_workspace_bytes(int64_t R, int C);
int csn_column_sum(const float* x, int64_t R, int C, float* out, void* workspace,
                   size_t workspace_bytes, void* stream);

/* Gate of GeometricGatedLinearUnit (python/clifford_model.py:42-43) on one GEMM output
 * gu [R, 2F] = [x W_gate^T | x W_up^T]:  y = silu(g) * u  [R, F];  backward dgu [R, 2F]. */
int csn_silu_gate_fwd(const float* gu, int64_t R, int F, float* y, void* stream);
int csn_silu_gate_bwd(const float* gu, const float* dy, int64_t R, int F, float* dgu, void* stream);

/* ------------------------------------------------- spatial blocks' generator chain */
/* The per-pixel chain of CliffordSpatialRotorBlockCl4 / Cl8 between their convolutions and
 * the Cayley rotor (csn_toolkit/csn/vision.py:79-94, :136-151), fused: from the NCHW outputs
 * in_proj [B, N*D*D, H, W], biv_proj [B, N*K, H, W] (K = D(D-1)/2, row-major triu) and
 * metric [B, N, H, W], with the parameters lambda_sw (1 value) and gamma_log [N] on the device,
 *   ds = softplus(metric), Omega = clamp((skew(biv) + tanh(lambda) (C - C^T) / 2) ds / 2, -3, 3),
 *   decay = sigmoid(-softplus(gamma_log) ds),
 * written pixel-major: omega, c [B, H*W, N, D, D], decay [B, H*W, N].  D in {4, 8, 16}.
 * The backward takes d_omega, d_c, d_decay in those layouts, writes the three NCHW input
 * gradients and per-CTA partial sums of dlambda [P] and dgamma [P, N], P =
 * csn_spatial_generators_partials(B, H*W, D) (0 for an unsupported D); the caller sums the
 * partials over P. */
int64_t csn_spatial_generators_partials(int64_t B, int64_t HW, int D);
int csn_spatial_generators_fwd(const float* in_proj, const float* biv_proj, const float* metric,
                               const float* lambda_sw, const float* gamma_log, float* omega, float* c,
                               float* decay, int64_t B, int64_t HW, int64_t N, int D, void* stream);
int csn_spatial_generators_bwd(const float* in_proj, const float* biv_proj, const float* metric,
                               const float* lambda_sw, const float* gamma_log, const float* d_omega,
                               const float* d_c, const float* d_decay, float* d_in_proj, float* d_biv_proj,
                               float* d_metric, float* dlambda_part, float* dgamma_part, int64_t B,
                               int64_t HW, int64_t N, int D, void* stream);

/* -------------------------------------------------------------- kernel timing */
/* Measurement hook with no counterpart in the reference (which times with wall clock,
 * tests/profile_performance.py:41-71).  While enabled, every kernel the library
 * launches is bracketed by a pair of CUDA events recorded on its own stream.
 * csn_timing_read() waits for those events and returns the summed elapsed time and
 * the launch count of kernels named `name` ("fwd_reduce", "fwd_carry", "fwd_apply",
 * "bwd_reduce", "bwd_carry", "bwd_apply", "reduce_channels"; NULL = all). */
int csn_timing_enable(int on);
int csn_timing_reset(void);
int csn_timing_read(const char* name, double* total_ms, int64_t* count);

#ifdef __cplusplus
}
#endif

#endif /* CSN_B200_H */
