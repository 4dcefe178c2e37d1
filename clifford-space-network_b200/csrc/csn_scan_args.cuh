// csn_scan_args.cuh -- argument block shared by the scan kernel families.
#pragma once

#include <stdint.h>

namespace csn {

// ----------------------------------------------------------------- arguments
struct ScanArgs {
  // plain scan inputs
  const float* M;
  const float* C;
  // fused rotor inputs
  const float* gens;
  const float* dt;
  const float* gamma;  // nullptr = undamped
  const float* S;
  // common
  const float* h0;  // [B, N, D, D] or nullptr
  const float* hT;  // backward: gradient entering after the last step, [B, N, D, D] or nullptr
  const float* X;   // forward output (backward only)
  const float* dX;  // incoming gradient (backward only)
  float* out;       // forward X
  // backward outputs
  float* dM;      // plain: dM     | rotor: unused
  float* dC;      // plain: dC     | rotor: dS
  float* dgens;   // rotor
  float* dgamma;  // rotor (damped)
  float* ddt_part;  // rotor: per (b, t, n) partial of ddt, reduced over n afterwards
  float* ddt;       // rotor: [B, T]
  float* dh0;       // [B, N, D, D] or nullptr
  // workspace
  float* aggP;   // [S, nchunks, D, D]
  float* aggC;   // [S, nchunks, D, D]
  float* carry;  // [S, nchunks, D, D]
  int64_t B, T, N;
  int64_t nchunks, chunk;
  // Sequence-parallel shard modes.
  //   agg_mode 1: reduce + compose, no apply pass; the chunk aggregates stay in aggP/aggC.
  //     forward:  P_out = M_{T-1} ... M_0, c_out = final state of a zero-carry scan
  //     backward: c_out = gradient leaving the shard at t = 0 with zero carry from t = T
  //   agg_mode 2: resume -- the chunk aggregates left by mode 1 on the same inputs are
  //     reused, so only the carry and apply passes run (carry-in h0; backward: hT).
  int agg_mode;
  float* P_out;  // [B, N, D, D]
  float* c_out;  // [B, N, D, D]
  int rev;       // plain scan in reverse time (X_t = M_t X_{t+1} (M_t^T) + C_t, X_T = h0)
  // Rotor cache (D = 16 fused scans): the step matrices M_t = sqrt(a_t) Q_t, [B, T, N, D, D].
  // A pass with Mc_out computes M_t and stores it; a pass with Mc_in loads it instead of
  // rebuilding the Cayley rotor.
  const float* Mc_in;
  float* Mc_out;
  // Backward: aggP already holds each chunk's product P_j (left there by the forward on the
  // same generators), so the backward reduce pass computes only the gradient aggregates.
  int reuse_P;
  // Per-head dt: with dtH > 1 the N channels are dtH heads of N / dtH neurons and dt (and
  // ddt) is [B, T, dtH]; channel n reads head n / (N / dtH).  0 or 1: dt is [B, T].
  int64_t dtH;
};

// Physical time of scan step t: the plain scan can run in reverse time (rev), i.e. scan
// step t reads and writes time T - 1 - t, so "the previous step" is the next time index.
__device__ __forceinline__ int64_t tphys(const ScanArgs& a, int64_t t) { return a.rev ? a.T - 1 - t : t; }

__device__ __forceinline__ int64_t elem(const ScanArgs& a, int64_t b, int64_t t, int64_t n) {
  return (b * a.T + tphys(a, t)) * a.N + n;
}

// Index of dt for batch b, physical time tp and channel n.
__device__ __forceinline__ int64_t dt_index(const ScanArgs& a, int64_t b, int64_t tp, int64_t n) {
  if (a.dtH <= 1) return b * a.T + tp;
  const uint32_t nh = static_cast<uint32_t>(a.N / a.dtH);  // N < 2^31 (checked by the entry points)
  return (b * a.T + tp) * a.dtH + static_cast<uint32_t>(n) / nh;
}

// Rows of the ddt reduction: ddt[b, t, h] = sum of the per-channel partials of head h.
__host__ __device__ __forceinline__ int64_t dt_heads(const ScanArgs& a) { return a.dtH > 1 ? a.dtH : 1; }

// ----------------------------------------------------------------- step sources
enum Src : int { SRC_MC = 0, SRC_ROTOR = 1 };

// Per-step rotor quantities kept for the backward pass.
template <int D, int K>
struct RotorStep {
  float g[K];
  float dt;
  float gamma;
  float alpha;
  float sa;  // sqrt(alpha)
};

}  // namespace csn
