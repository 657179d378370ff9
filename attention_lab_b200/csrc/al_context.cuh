// Kernels of the context split across GPUs (config C4): positions [0, L) are split into P contiguous shards, each
// rank takes a local top-k of its candidates (the fused kernel in select-only mode, with 64-bit candidate keys),
// the ranks all-gather those keys, every rank finds the global k-th key here and attends over its own chosen rows
// into an unnormalised partial (m, l, acc), and the all-gathered partials are merged by log-sum-exp. The chosen set
// equals the single-device top-k exactly: a 64-bit key holds the score's order key above the inverted position, so
// (score desc, position asc) is plain 64-bit order and no two real candidates tie.
#pragma once
#include "al_decode.cuh"

namespace al {

// ------------------------------------------------------------------------------------------------ peer exchange
// The ranks' exchange regions (one cudaMalloc'd region per GPU, mapped by the others through CUDA IPC) replace the two
// NCCL all-gathers. A channel (keys, partials) has in every region a gather area with one slot per rank, a flag word
// per rank and an epoch counter. xchg_push_kernel copies this rank's data into its slot of every rank's gather area
// (stores over NVLink, which do not stall the copying threads), and the last CTA to finish advances this rank's epoch
// and stores it into every peer's flag for this rank (system-scope fences before the release stores: the data is
// visible first). A consumer waits for every peer's flag to reach its own epoch (system-scope acquire, bounded: a wait
// that gives up sets kErrWaitLimit and the launch's results are invalid) and reads only its own gather area. The
// epoch lives on the device, so a captured CUDA graph replays with fresh epochs. A rank pushes into a slot again only
// after a later step that needed every peer's data, so one slot per rank and channel suffices.
struct XchgWait {
  const unsigned* flags;            // this rank's flags of the channel: flags[q] is written by rank q
  const unsigned* counter;          // this rank's epoch counter of the channel (set by its push)
  int P, rank, spin;                // spin: polls of one peer's flag before giving up
  unsigned* err;
};

// Thread 0 of a CTA: wait until every peer's flag has reached this rank's epoch.
__device__ __forceinline__ void xchg_wait(const XchgWait& w) {
  const unsigned e = *reinterpret_cast<const volatile unsigned*>(w.counter);
  for (int q = 0; q < w.P; ++q) {
    if (q == w.rank) continue;
    for (int it = 0;; ++it) {
      unsigned f;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(f) : "l"(w.flags + q) : "memory");
      if ((int)(f - e) >= 0) break;
      if (it >= w.spin) { atomicOr(w.err, kErrWaitLimit); break; }
      __nanosleep(128);
    }
  }
}

struct XchgPush {
  const int4* src;                  // this rank's data (n16 16-byte words)
  long long n16;
  int4* const* dst;                 // [P] the ranks' gather areas of the channel; this rank's slot at + rank * n16
  int P, rank;
  unsigned* done;                   // CTAs finished with the copy (this rank's region; reset by the last one)
  unsigned* counter;                // this rank's epoch counter of the channel
  unsigned* const* peer_flags;      // [P] the ranks' flag arrays of the channel
};

__global__ void __launch_bounds__(256) xchg_push_kernel(const XchgPush x) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < x.n16; i += stride) {
    const int4 v = x.src[i];
    for (int q = 0; q < x.P; ++q) x.dst[q][(long long)x.rank * x.n16 + i] = v;
  }
  __threadfence_system();
  __syncthreads();
  __shared__ bool s_last;
  if (threadIdx.x == 0) s_last = atomicAdd(x.done, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!s_last || threadIdx.x != 0) return;
  *x.done = 0u;
  __threadfence_system();
  const unsigned e = *x.counter + 1u;
  *x.counter = e;
  for (int q = 0; q < x.P; ++q)
    if (q != x.rank) asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(x.peer_flags[q] + x.rank), "r"(e) : "memory");
}

struct CtxParams {
  int P, B, G, kst, k, rank, F, k_local;
  const unsigned long long* keys;   // [P, B, G, kst] all ranks' keys (zero padding below every real key)
  const long long* rows_in;         // [B, G, F + k_local] this rank's rows: F, then its candidates in key order
  long long* rows_attend;           // [B, G, F + k_local] the same rows, -1 where a candidate is not in the top-k
  // peer exchange (wait.flags non-null): `keys` is this rank's gather area, filled by the ranks' pushes; the CTA waits
  // for every peer's flag first
  XchgWait wait;
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
  if (p.wait.flags) {
    if (tid == 0) xchg_wait(p.wait);
    __syncthreads();
  }
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

// The same merge over this rank's gather area of partials, filled by the ranks' pushes, after a bounded wait for every
// peer's flag by thread 0 of each block.
template <typename T>
__global__ void __launch_bounds__(256) lse_merge_wait_kernel(const float* __restrict__ parts, XchgWait w, int n,
                                                              T* __restrict__ out) {
  if (threadIdx.x == 0) xchg_wait(w);
  __syncthreads();
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n * kHeadDim) return;
  const int row = idx / kHeadDim, d = idx % kHeadDim;
  float M = -INFINITY;
  for (int q = 0; q < w.P; ++q) {
    const float* pp = parts + ((size_t)q * n + row) * (kHeadDim + 2);
    if (pp[1] > 0.f) M = fmaxf(M, pp[0]);
  }
  float L = 0.f, A = 0.f;
  for (int q = 0; q < w.P; ++q) {
    const float* pp = parts + ((size_t)q * n + row) * (kHeadDim + 2);
    if (pp[1] > 0.f) {
      const float wq = exp2f(pp[0] - M);
      L = fmaf(wq, pp[1], L);
      A = fmaf(wq, pp[2 + d], A);
    }
  }
  out[idx] = fromf<T>(A / L);
}

}  // namespace al
