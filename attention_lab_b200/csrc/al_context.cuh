// Kernels of the context split across GPUs (config C4): positions [0, L) are split into P contiguous shards, each
// rank takes a local top-k of its candidates (the fused kernel in select-only mode, with 64-bit candidate keys),
// the ranks all-gather those keys, every rank finds the global k-th key here and attends over its own chosen rows
// into an unnormalised partial (m, l, acc), and the all-gathered partials are merged by log-sum-exp. The chosen set
// equals the single-device top-k exactly: a 64-bit key holds the score's order key above the inverted position, so
// (score desc, position asc) is plain 64-bit order and no two real candidates tie.
#pragma once
#include "al_decode.cuh"

namespace al {

struct CtxParams {
  int P, B, G, kst, k, rank, F, k_local;
  const unsigned long long* keys;   // [P, B, G, kst] all ranks' keys (zero padding below every real key)
  const long long* rows_in;         // [B, G, F + k_local] this rank's rows: F, then its candidates in key order
  long long* rows_attend;           // [B, G, F + k_local] the same rows, -1 where a candidate is not in the top-k
};

// One CTA per (batch, group) segment: a radix select over the P * kst keys (six digits of 11/11/11/11/10/10 bits,
// block histograms, the keys read from L2) finds the k-th largest 64-bit key tau; this rank keeps its candidates
// with key >= tau. Reference: the global top-k of decode.py:92 over the union of the shards' candidates.
__global__ void __launch_bounds__(kThreads) context_threshold_kernel(const CtxParams p) {
  __shared__ unsigned s_hist[2048];
  __shared__ int s_sltot[kMaxCluster], s_piv[2], s_ws[kWarps];
  cg::cluster_group cluster = cg::this_cluster();
  const int seg = blockIdx.x, tid = threadIdx.x;
  if (tid == 0) { s_piv[0] = 0; s_piv[1] = 0; }
  const int BG = p.B * p.G, N = p.P * p.kst;
  auto key_at = [&](int j) { return p.keys[((size_t)(j / p.kst) * BG + seg) * p.kst + (j % p.kst)]; };
  unsigned long long prefix = 0ull, pmask = 0ull;
  int need = p.k;
  const int shifts[6] = {53, 42, 31, 20, 10, 0};
  const int widths[6] = {11, 11, 11, 11, 10, 10};
#pragma unroll 1
  for (int d = 0; d < 6; ++d) {
    const int sh = shifts[d], nb = 1 << widths[d];
    for (int i = tid; i < 2048; i += kThreads) s_hist[i] = 0u;
    __syncthreads();
    for (int j = tid; j < N; j += kThreads) {
      const unsigned long long kv = key_at(j);
      if ((kv & pmask) == prefix) atomicAdd(&s_hist[(unsigned)(kv >> sh) & (unsigned)(nb - 1)], 1u);
    }
    __syncthreads();
    int bin, above;
    pivot_round(cluster, 1, 0, s_hist, nullptr, s_sltot, s_piv, s_ws, nb, need, bin, above);
    prefix |= (unsigned long long)bin << sh;
    pmask |= (unsigned long long)(nb - 1) << sh;
    need -= above;
  }
  const unsigned long long tau = prefix;
  const int S = p.F + p.k_local;
  const long long* ri = p.rows_in + (size_t)seg * S;
  long long* ra = p.rows_attend + (size_t)seg * S;
  for (int i = tid; i < S; i += kThreads) {
    long long row = ri[i];
    if (i >= p.F && key_at(p.rank * p.kst + (i - p.F)) < tau) row = -1;
    ra[i] = row;
  }
}

// out[b,g,head,:] = sum_p 2^(m_p - M) acc_p / sum_p 2^(m_p - M) l_p over the P partials (m in the log2 domain,
// M the largest m of a non-empty partial). The LSE combine of the reference's partitioned attend
// (metal_attend.py:147-169).
template <typename T>
__global__ void __launch_bounds__(256) lse_merge_kernel(const float* __restrict__ parts, int P, int n, T* __restrict__ out) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n * kHeadDim) return;
  const int row = idx / kHeadDim, d = idx % kHeadDim;
  float M = -INFINITY;
  for (int q = 0; q < P; ++q) {
    const float* pp = parts + ((size_t)q * n + row) * (kHeadDim + 2);
    if (pp[1] > 0.f) M = fmaxf(M, pp[0]);
  }
  float L = 0.f, A = 0.f;
  for (int q = 0; q < P; ++q) {
    const float* pp = parts + ((size_t)q * n + row) * (kHeadDim + 2);
    if (pp[1] > 0.f) {
      const float w = exp2f(pp[0] - M);
      L = fmaf(w, pp[1], L);
      A = fmaf(w, pp[2 + d], A);
    }
  }
  out[idx] = fromf<T>(A / L);
}

}  // namespace al
