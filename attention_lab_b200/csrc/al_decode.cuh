// The fused sparse decode step: one kernel launch per layer does the whole D chain of
// attention-lab's decode.py:145-163 for every (batch, group) segment:
//
//   z of the newest key into zT[..., write_col]   (decode.py:156-157, indexer.py:15-17)
//   u = concat_h(q_pre) . wq_t_scaled             (indexer.py:20-24)
//   s = u . zT[..., lo:hi]                         (indexer.py:27-29)   16-byte streamed loads, fp32 accumulate
//   top-k of s with ties to the smaller position   (decode.py:92)        3-pass radix select on order keys
//   rows = F ++ chosen candidates                  (decode.py:93)        optionally ascending (decode.py:160-161)
//   attention over exactly those rows              (decode.py:131-142)   gather-free, rows read in place
//
// A segment is served by a thread-block cluster of CS CTAs (CS in 1..16). CTA c owns a contiguous slice of the
// candidate columns; its scores stay in its shared memory as order keys. The radix histograms are reduce-scattered
// across the cluster through distributed shared memory, so the segment's exact k-th key is found without any global
// scratch. Each CTA then attends over the candidates it selected plus a share of F, and the cluster merges the
// partial softmax states (log-sum-exp) into the output. Nothing is written to global memory except the z column,
// the output, and the optional row list and scores.
#pragma once
#include "al_attend.cuh"

namespace al {

struct DecodeParams {
  int B, G, h, r, C;
  int lo, hi, M, k, S, F, write_col;
  int select_mode;        // 0: no candidate (k == 0); 1: radix top-k; 2: every candidate (k == M)
  int scan;               // 1: compute scores (select_mode 1 or scores requested)
  int zvec;               // 1: 16-byte aligned zT rows (C * sizeof(idx) % 16 == 0 and aligned base)
  int uvec;               // 1: r == 32 and 16-byte aligned wq_t (vector u prologue)
  int canonical;
  int cpc;                // candidate columns per CTA (a multiple of 8)
  int union_bytes;        // bytes of the [keys | candidate list] / attend-engine union at the start of dynamic smem
  int keys_bytes;         // bytes of the key array (the candidate list follows it)
  int ccap;               // candidate-list capacity per CTA (entries)
  int nstage;             // attend pipeline depth (4..8)
  float scale_log2;
  long long total_rows;   // B*G*C rows in the flattened cache
  const void* q; long long q_sb, q_sg, q_sh;        // q_main [B,G,h,1,d], KV dtype
  const void* q_pre; long long qp_sb, qp_sg, qp_sh; // q_pre [B,G,h,1,d], index dtype (unused when u_in is given)
  const void* u_in;                                 // u [B,G,r], index dtype (select_rows_kernel input), nullable
  const void* wq_t;                                 // [G, h*d, r]
  const void* wk;                                   // [G, r, d]
  const void* k_new; long long kn_sb, kn_sg;        // k_pre_new [B,G,1,d], nullable
  void* zT;                                         // [B,G,r,C]
  const void* k_cache; const void* v_cache;         // [B,G,C,d]
  const long long* fixed_rows;                      // [B,G,F] flat rows
  const long long* off_lo;                          // [B,G,1] flat row of candidate 0
  void* out;                                        // [B,G,h,d], nullable: select only
  float* part;                                      // [B,G,h,130] partial (m, l, acc) instead of out, nullable
  long long* rows_out;                              // [B,G,S], nullable
  float* scores_out;                                // [B,G,M], nullable
  unsigned* err;                                    // device error word
};

__device__ __forceinline__ uint32_t checked_row(long long row, long long total, unsigned* err) {
  if (row < 0 || row >= total) {
    atomicOr(err, kErrRowRange);
    return 0xffffffffu;
  }
  return (uint32_t)row;
}

// u = concat_h(q_pre) . wq_t  (or the given u) into s_u[0..32), zero-padded beyond r.
// Vector path (r == 32, 16-byte aligned weights): a thread owns VW adjacent j of one f row per iteration (16-byte
// weight loads, all independent), then the f partial sums are reduced by shuffles within the warp and through
// shared memory across warps.
template <typename IDX_T>
__device__ void compute_u(const DecodeParams& p, int b, int g, float* s_u, float* s_pre) {
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5, seg = b * p.G + g;
  if (p.u_in) {
    if (tid < kMaxR) s_u[tid] = (tid < p.r) ? tof(reinterpret_cast<const IDX_T*>(p.u_in)[(size_t)seg * p.r + tid]) : 0.f;
    __syncthreads();
    return;
  }
  const IDX_T* qp = reinterpret_cast<const IDX_T*>(p.q_pre) + b * p.qp_sb + g * p.qp_sg;
  const int hd = p.h * kHeadDim;
  const IDX_T* wq = reinterpret_cast<const IDX_T*>(p.wq_t) + (size_t)g * hd * p.r;
  if (p.uvec) {
    constexpr int VW = V16<IDX_T>::n;
    constexpr int TPR = kMaxR / VW;                     // threads per f row
    constexpr int RPI = kThreads / TPR;                 // f rows per iteration
    const int jg = tid % TPR, fr = tid / TPR;
    float acc[VW];
#pragma unroll
    for (int e = 0; e < VW; ++e) acc[e] = 0.f;
#pragma unroll 4
    for (int f = fr; f < hd; f += RPI) {
      const uint4 v = *reinterpret_cast<const uint4*>(wq + (size_t)f * kMaxR + jg * VW);
      const float qv = tof(qp[(f / kHeadDim) * p.qp_sh + (f % kHeadDim)]);
      float wv[VW];
      unpack(v, wv, (const IDX_T*)nullptr);
#pragma unroll
      for (int e = 0; e < VW; ++e) acc[e] = fmaf(qv, wv[e], acc[e]);
    }
#pragma unroll
    for (int o = TPR; o < 32; o <<= 1)
#pragma unroll
      for (int e = 0; e < VW; ++e) acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], o);
    if (lane < TPR) {
#pragma unroll
      for (int e = 0; e < VW; ++e) s_pre[w * 32 + lane * VW + e] = acc[e];
    }
  } else {
    const int j = lane;
    float acc = 0.f;
    if (j < p.r)
      for (int f = w; f < hd; f += kWarps)
        acc = fmaf(tof(qp[(f / kHeadDim) * p.qp_sh + (f % kHeadDim)]), tof(wq[(size_t)f * p.r + j]), acc);
    s_pre[w * 32 + j] = acc;
  }
  __syncthreads();
  if (tid < kMaxR) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kWarps; ++i) s += s_pre[i * 32 + tid];
    s_u[tid] = (tid < p.r) ? s : 0.f;
  }
  __syncthreads();
}

// z of the newest key: zT[b,g,j,write_col] = sum_e wk[g,j,e] * k_new[b,g,e], rounded to the index dtype.
template <typename IDX_T>
__device__ void write_z_column(const DecodeParams& p, int b, int g) {
  static_assert(kThreads == 16 * kMaxR, "one 16-lane group per index row");
  const int tid = threadIdx.x, j = tid >> 4, part = tid & 15, seg = b * p.G + g;
  const IDX_T* kn = reinterpret_cast<const IDX_T*>(p.k_new) + b * p.kn_sb + g * p.kn_sg;
  const IDX_T* wk = reinterpret_cast<const IDX_T*>(p.wk) + ((size_t)g * p.r + (j < p.r ? j : 0)) * kHeadDim;
  float acc = 0.f;
  if (j < p.r) {
#pragma unroll
    for (int e = part * 8; e < part * 8 + 8; ++e) acc = fmaf(tof(wk[e]), tof(kn[e]), acc);
  }
  acc += __shfl_xor_sync(0xffffffffu, acc, 1);
  acc += __shfl_xor_sync(0xffffffffu, acc, 2);
  acc += __shfl_xor_sync(0xffffffffu, acc, 4);
  acc += __shfl_xor_sync(0xffffffffu, acc, 8);
  if (j < p.r && part == 0)
    reinterpret_cast<IDX_T*>(p.zT)[((size_t)seg * p.r + j) * p.C + p.write_col] = fromf<IDX_T>(acc);
}

// Scores of candidate columns [c0, c1) -> order keys. The key of column c is stored at s_keys[c - kbase] with
// kbase = c0 rounded down to a multiple of 8, so every 16-byte group of keys is aligned; indices outside
// [c0 - kbase, c1 - kbase) hold no valid key. When s_hist is given, also counts every valid key's top 12 bits into
// it (the first radix digit, hidden under the scan's memory latency), and writes fp32 scores when requested. Vector path: each thread owns VW adjacent columns and streams all r rows of them with
// 16-byte loads (8 or 16 rows in flight); u is read from shared memory as broadcast float4s.
template <typename IDX_T>
__device__ void scan_columns(const DecodeParams& p, int seg, int c0, int c1, int kbase, const float* s_u,
                             uint32_t* s_keys, unsigned* s_hist) {
  const IDX_T* zseg = reinterpret_cast<const IDX_T*>(p.zT) + (size_t)seg * p.r * p.C;
  float* so = p.scores_out ? p.scores_out + (size_t)seg * p.M - p.lo : nullptr;   // indexed by column
  if (p.zvec) {
    constexpr int VW = V16<IDX_T>::n;
    constexpr int RB = 16;                                   // rows in flight per thread (64 load registers)
    const int a0 = (c0 / VW) * VW;
    const int ngr = (c1 - a0 + VW - 1) / VW;
    const float4* u4 = reinterpret_cast<const float4*>(s_u);
#pragma unroll 1
    for (int gi = threadIdx.x; gi < ngr; gi += kThreads) {
      const int col = a0 + gi * VW;
      const IDX_T* zc = zseg + col;
      float2 acc2[VW / 2];
#pragma unroll
      for (int e = 0; e < VW / 2; ++e) acc2[e] = make_float2(0.f, 0.f);
#pragma unroll
      for (int jb = 0; jb < kMaxR; jb += RB) {
        uint4 v[RB];
#pragma unroll
        for (int jj = 0; jj < RB; ++jj)
          v[jj] = (jb + jj < p.r) ? ldg_stream16(zc + (size_t)(jb + jj) * p.C) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
        for (int jq = 0; jq < RB; jq += 4) {
          const float4 uu = u4[(jb + jq) / 4];
          const float uj[4] = {uu.x, uu.y, uu.z, uu.w};
#pragma unroll
          for (int x = 0; x < 4; ++x) {
            float f[VW];
            unpack(v[jq + x], f, (const IDX_T*)nullptr);
            const float2 u2 = make_float2(uj[x], uj[x]);
#pragma unroll
            for (int e = 0; e < VW / 2; ++e) acc2[e] = __ffma2_rn(u2, make_float2(f[2 * e], f[2 * e + 1]), acc2[e]);
          }
        }
      }
      float acc[VW];
#pragma unroll
      for (int e = 0; e < VW / 2; ++e) { acc[2 * e] = acc2[e].x; acc[2 * e + 1] = acc2[e].y; }
      uint32_t kk[VW];
#pragma unroll
      for (int e = 0; e < VW; ++e) {
        kk[e] = score_key(acc[e]);
        const int c = col + e;
        if (c >= c0 && c < c1) {
          if (s_hist) atomicAdd(&s_hist[kk[e] >> 20], 1u);
          if (so) so[c] = acc[e];
        }
      }
#pragma unroll
      for (int e = 0; e < VW; e += 4)
        *reinterpret_cast<uint4*>(s_keys + (col - kbase) + e) = make_uint4(kk[e], kk[e + 1], kk[e + 2], kk[e + 3]);
    }
  } else {
    for (int c = c0 + threadIdx.x; c < c1; c += kThreads) {
      float a = 0.f;
      for (int j = 0; j < p.r; ++j) a = fmaf(s_u[j], tof(zseg[(size_t)j * p.C + c]), a);
      const uint32_t key = score_key(a);
      s_keys[c - kbase] = key;
      if (s_hist) atomicAdd(&s_hist[key >> 20], 1u);
      if (so) so[c] = a;
    }
  }
}

// Cluster-wide pivot search over the CTAs' NB-bin histograms (complete and visible cluster-wide on entry): the bin
// holding the need-th largest element counted from the top bin, and the number of elements in the bins above it.
// Every CTA returns the same result. CS == 1 uses block barriers only.
__device__ void pivot_round(cg::cluster_group& cluster, int CS, int crank, const unsigned* s_hist, unsigned* s_slice,
                            int* s_sltot, int* s_piv, int* s_ws, int NB, int need, int& bin_out, int& above_out) {
  const int tid = threadIdx.x;
  const int SL = NB / CS, s0 = crank * SL;
  for (int i = tid; i < SL; i += kThreads) {
    unsigned v = 0;
    if (CS == 1) v = s_hist[i];
    else
      for (int c = 0; c < CS; ++c) v += cluster.map_shared_rank(s_hist, c)[s0 + i];
    s_slice[i] = v;
  }
  __syncthreads();
  const int BPT = (SL + kThreads - 1) / kThreads;
  int lsum = 0;
  for (int i = 0; i < BPT; ++i) {
    const int bin = tid * BPT + i;
    if (bin < SL) lsum += (int)s_slice[bin];
  }
  int tot;
  const int incl = block_inclusive_scan(lsum, s_ws, &tot);
  int cum = 0, ps = 0;
  if (CS > 1) {
    if (tid < CS) cluster.map_shared_rank(s_sltot, tid)[crank] = tot;
    cluster.sync();
    ps = -1;
    for (int c = CS - 1; c >= 0; --c) {
      const int t2 = s_sltot[c];
      if (cum + t2 >= need) { ps = c; break; }
      cum += t2;
    }
  }
  if (ps == crank) {
    const int nd = need - cum;
    int above = tot - incl;
    for (int i = BPT - 1; i >= 0; --i) {
      const int bin = tid * BPT + i;
      if (bin < SL) {
        const int hv = (int)s_slice[bin];
        if (above < nd && above + hv >= nd) {
          if (CS == 1) { s_piv[0] = s0 + bin; s_piv[1] = cum + above; }
          else
            for (int c = 0; c < CS; ++c) {
              int* pp = cluster.map_shared_rank(s_piv, c);
              pp[0] = s0 + bin;
              pp[1] = cum + above;
            }
        }
        above += hv;
      }
    }
  }
  if (CS > 1) cluster.sync(); else __syncthreads();
  bin_out = s_piv[0];
  above_out = s_piv[1];
}

template <typename KV_T, typename IDX_T, int HP>
__global__ void __launch_bounds__(kThreads, 1) sparse_step_kernel(const DecodeParams p) {
  extern __shared__ __align__(128) unsigned char dsm[];
  __shared__ __align__(16) float s_u[kMaxR];
  __shared__ float s_pre[kWarps * 32];
  __shared__ unsigned s_hist[4096];
  __shared__ unsigned s_slice[4096];
  __shared__ int s_sltot[kMaxCluster];
  __shared__ int s_cgt[kMaxCluster], s_ceq[kMaxCluster], s_cflag[kMaxCluster];
  __shared__ int s_piv[2];
  __shared__ int s_ws[kWarps];
  __shared__ int s_fpre;
  __shared__ float s_m[HP], s_l[HP];
  __shared__ float s_acc[HP * kHeadDim];

  cg::cluster_group cluster = cg::this_cluster();
  const int CS = (int)cluster.num_blocks();
  const int crank = (int)cluster.block_rank();
  const int seg = blockIdx.y;
  const int b = seg / p.G, g = seg - b * p.G;
  const int tid = threadIdx.x;
  // dynamic shared memory: [keys | candidate list] aliasing [attend engine], then the attend row list
  uint32_t* s_keys = reinterpret_cast<uint32_t*>(dsm);
  uint32_t* cand_key = reinterpret_cast<uint32_t*>(dsm + p.keys_bytes);
  uint32_t* cand_idx = cand_key + p.ccap;
  uint32_t* s_arow = reinterpret_cast<uint32_t*>(dsm + p.union_bytes);
#define CSYNC() do { if (CS > 1) cluster.sync(); else __syncthreads(); } while (0)

  // ---------------- prologue: z column (rank 0 of the cluster) and u ----------------
  if (p.select_mode == 1)
    for (int i = tid; i < 4096; i += kThreads) s_hist[i] = 0u;
  if (p.k_new && crank == 0) write_z_column<IDX_T>(p, b, g);
  if (p.scan) compute_u<IDX_T>(p, b, g, s_u, s_pre);

  const int c0 = p.lo + crank * p.cpc;
  const int c1 = min(p.hi, c0 + p.cpc);
  const int nloc = max(0, c1 - c0);
  const int kbase = (c0 / 8) * 8, koff = c0 - kbase;

  // ---------------- scan: candidate scores -> order keys, plus the histogram of their top 12 bits ----------------
  if (p.scan && nloc > 0)
    scan_columns<IDX_T>(p, seg, c0, c1, kbase, s_u, s_keys, p.select_mode == 1 ? s_hist : nullptr);
  CSYNC();

  // key quads [q0, q1) cover the valid key indices [koff, koff + nloc); thread runs use an odd stride so the 8
  // threads of a quarter warp read 8 different bank groups
  const int q0 = koff / 4, q1 = (koff + nloc + 3) / 4;
  const int QPT = (((q1 - q0) + kThreads - 1) / kThreads) | 1;
  const int tq0 = min(q1, q0 + tid * QPT), tq1 = min(q1, tq0 + QPT);
  const uint4* keys4 = reinterpret_cast<const uint4*>(s_keys);

  // ---------------- radix select of the k-th largest key over the cluster ----------------
  // 1) the histogram of the top 12 key bits (built during the scan) gives the pivot bin b0;
  // 2) one ordered pass copies every key with top bits >= b0 into a short candidate list (k plus the pivot bin);
  // 3) two 10-bit passes over the list's pivot-bin keys find the exact k-th key tau and how many of its copies
  //    (k_rem, in position order) complete the top-k. If some CTA's list would overflow, steps 2-3 run over the
  //    full key array instead.
  uint32_t tau = 0;
  int k_rem = 0;
  bool use_list = false;
  int n_cand = 0;
  if (p.select_mode == 1) {
    int b0, gt0;
    pivot_round(cluster, CS, crank, s_hist, s_slice, s_sltot, s_piv, s_ws, 4096, p.k, b0, gt0);
    const int need0 = p.k - gt0;
    // candidate count of this thread's run, then its offset in the CTA's list
    int cnt = 0;
    for (int qi = tq0; qi < tq1; ++qi) {
      const uint4 k4 = keys4[qi];
      const uint32_t kv[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int idx = qi * 4 + e;
        cnt += (idx >= koff && idx < koff + nloc && (int)(kv[e] >> 20) >= b0) ? 1 : 0;
      }
    }
    int ctot;
    const int cinc = block_inclusive_scan(cnt, s_ws, &ctot);
    if (CS > 1) {
      if (tid < CS) cluster.map_shared_rank(s_cflag, tid)[crank] = ctot > p.ccap ? 1 : 0;
      cluster.sync();
      use_list = true;
      for (int c = 0; c < CS; ++c) use_list = use_list && s_cflag[c] == 0;
    } else {
      use_list = ctot <= p.ccap;
    }
    if (use_list) {
      int o = cinc - cnt;
      for (int qi = tq0; qi < tq1; ++qi) {
        const uint4 k4 = keys4[qi];
        const uint32_t kv[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int idx = qi * 4 + e;
          if (idx >= koff && idx < koff + nloc && (int)(kv[e] >> 20) >= b0) {
            cand_key[o] = kv[e];
            cand_idx[o] = (uint32_t)idx;
            ++o;
          }
        }
      }
      n_cand = ctot;
    }
    // refinement over the keys of bin b0: bits 19..10, then 9..0
    uint32_t prefix = (uint32_t)b0 << 20, pmask = 0xfff00000u;
    k_rem = need0;
#pragma unroll 1
    for (int pass = 0; pass < 2; ++pass) {
      const int shift = pass == 0 ? 10 : 0;
      for (int i = tid; i < 1024; i += kThreads) s_hist[i] = 0u;
      __syncthreads();
      if (use_list) {
        for (int i = tid; i < n_cand; i += kThreads) {
          const uint32_t key = cand_key[i];
          if ((key & pmask) == prefix) atomicAdd(&s_hist[(key >> shift) & 1023u], 1u);
        }
      } else {
        for (int qi = tq0; qi < tq1; ++qi) {
          const uint4 k4 = keys4[qi];
          const uint32_t kv[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int idx = qi * 4 + e;
            if (idx >= koff && idx < koff + nloc && (kv[e] & pmask) == prefix)
              atomicAdd(&s_hist[(kv[e] >> shift) & 1023u], 1u);
          }
        }
      }
      CSYNC();
      int bn, above;
      pivot_round(cluster, CS, crank, s_hist, s_slice, s_sltot, s_piv, s_ws, 1024, k_rem, bn, above);
      prefix |= (uint32_t)bn << shift;
      pmask |= 1023u << shift;
      k_rem -= above;
    }
    tau = prefix;
  }

  // ---------------- ordered selection: chosen candidates in ascending position order ----------------
  const long long seg_off = p.off_lo[seg];
  const int F = p.F;
  const int fsh0 = (crank * F) / CS, fsh1 = ((crank + 1) * F) / CS, fshare = fsh1 - fsh0;
  if (tid == 0) {
    int fp = 0;
    if (p.canonical)
      for (int i = 0; i < F; ++i) fp += (p.fixed_rows[(size_t)seg * F + i] < seg_off) ? 1 : 0;
    s_fpre = fp;
  }
  int n_sel = 0;
  if (p.select_mode != 0) {
    const bool all = p.select_mode == 2;
    // this thread's entries: a run of the candidate list, or its run of key quads
    const int EPT = ((n_cand + kThreads - 1) / kThreads) | 1;
    const int te0 = min(n_cand, tid * EPT), te1 = min(n_cand, te0 + EPT);
    int cgt = 0, ceq = 0;
    if (use_list) {
      for (int i = te0; i < te1; ++i) {
        const uint32_t key = cand_key[i];
        cgt += key > tau ? 1 : 0;
        ceq += key == tau ? 1 : 0;
      }
    } else {
      for (int qi = tq0; qi < tq1; ++qi) {
        uint4 k4 = make_uint4(0u, 0u, 0u, 0u);
        if (!all) k4 = keys4[qi];
        const uint32_t kv[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int idx = qi * 4 + e;
          const bool in = idx >= koff && idx < koff + nloc;
          cgt += (in && (all || kv[e] > tau)) ? 1 : 0;
          ceq += (in && !all && kv[e] == tau) ? 1 : 0;
        }
      }
    }
    // packed block scan of (gt, eq) counts: both stay below 2^16 per CTA
    const unsigned packed = (unsigned)cgt | ((unsigned)ceq << 16);
    int tot;
    const unsigned inc = (unsigned)block_inclusive_scan((int)packed, s_ws, &tot);
    const int ex_gt = (int)((inc - packed) & 0xffffu), ex_eq = (int)((inc - packed) >> 16);
    const int tot_gt = (int)((unsigned)tot & 0xffffu), tot_eq = (int)((unsigned)tot >> 16);
    int eo = 0, so = 0;                         // ties and selections before this CTA
    if (CS > 1) {
      if (tid < CS) {
        cluster.map_shared_rank(s_cgt, tid)[crank] = tot_gt;
        cluster.map_shared_rank(s_ceq, tid)[crank] = tot_eq;
      }
      cluster.sync();
      for (int c = 0; c < crank; ++c) { so += s_cgt[c]; eo += s_ceq[c]; }
      so += min(max(k_rem, 0), eo);
    }
    const int sel_off = so;                     // this CTA's first rank
    n_sel = tot_gt + min(max(k_rem - eo, 0), tot_eq);
    int er = eo + ex_eq;                        // tie rank of this thread's first equal key
    int rank = so + ex_gt + min(max(k_rem - eo, 0), ex_eq);
    const int out_base = p.canonical ? s_fpre : F;
    long long* ro = p.rows_out ? p.rows_out + (size_t)seg * p.S + out_base : nullptr;
    auto emit = [&](int idx) {
      const long long row = seg_off + (long long)(kbase + idx - p.lo);
      if (ro) ro[rank] = row;
      s_arow[fshare + (rank - sel_off)] = checked_row(row, p.total_rows, p.err);
      ++rank;
    };
    if (use_list) {
      for (int i = te0; i < te1; ++i) {
        const uint32_t key = cand_key[i];
        if (key > tau) emit((int)cand_idx[i]);
        else if (key == tau) {
          if (er < k_rem) emit((int)cand_idx[i]);
          ++er;
        }
      }
    } else {
      for (int qi = tq0; qi < tq1; ++qi) {
        uint4 k4 = make_uint4(0u, 0u, 0u, 0u);
        if (!all) k4 = keys4[qi];
        const uint32_t kv[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int idx = qi * 4 + e;
          if (!(idx >= koff && idx < koff + nloc)) continue;
          if (all || kv[e] > tau) emit(idx);
          else if (kv[e] == tau) {
            if (er < k_rem) emit(idx);
            ++er;
          }
        }
      }
    }
  }
  for (int i = tid; i < fshare; i += kThreads)
    s_arow[i] = checked_row(p.fixed_rows[(size_t)seg * F + fsh0 + i], p.total_rows, p.err);
  __syncthreads();
  if (p.rows_out && crank == 0 && tid < 32) {
    // F into the row list: first (reference order), or around the candidates when canonical
    const int lane = tid;
    long long* ro = p.rows_out + (size_t)seg * p.S;
    const long long* fr = p.fixed_rows + (size_t)seg * F;
    if (!p.canonical) {
      for (int i = lane; i < F; i += 32) ro[i] = fr[i];
    } else {
      int nlo = 0, nhi = 0;
      const unsigned lt = (1u << lane) - 1u;
      for (int base = 0; base < F; base += 32) {
        const int i = base + lane;
        const long long v = i < F ? fr[i] : 0;
        const bool lo_side = i < F && v < seg_off, hi_side = i < F && v >= seg_off;
        const unsigned ml = __ballot_sync(0xffffffffu, lo_side), mh = __ballot_sync(0xffffffffu, hi_side);
        if (lo_side) ro[nlo + __popc(ml & lt)] = v;
        if (hi_side) ro[s_fpre + p.k + nhi + __popc(mh & lt)] = v;
        nlo += __popc(ml);
        nhi += __popc(mh);
      }
    }
  }
  if (!p.out && !p.part) {
    if (CS > 1) cluster.sync();   // peers may still read this CTA's counters
    return;
  }
#undef CSYNC

  // ---------------- attend over this CTA's rows, then the cluster merge ----------------
  const float* s_q = stage_q<KV_T, HP>(dsm, p.nstage, reinterpret_cast<const KV_T*>(p.q) + b * p.q_sb + g * p.q_sg,
                                      p.q_sh, p.h);
  __syncthreads();
  RowSrc rs{s_arow, 0u};
  attend_rows<KV_T, HP>(reinterpret_cast<const KV_T*>(p.k_cache), reinterpret_cast<const KV_T*>(p.v_cache), rs,
                        fshare + n_sel, s_q, p.scale_log2, dsm, p.nstage, s_m, s_l, s_acc);
  finish_output<KV_T, HP>(p.out ? reinterpret_cast<KV_T*>(p.out) + (size_t)seg * p.h * kHeadDim : nullptr,
                          p.part ? p.part + (size_t)seg * p.h * (kHeadDim + 2) : nullptr, p.h, s_m, s_l, s_acc);
}

// ------------------------------------------------------------------------------------------------ attend only
struct AttendParams {
  int B, G, h, C, S, L;
  int mode;               // 0: gathered rows [B,G,S] flat ids; 1: dense range [0, L) of each segment
  int rows_cap;
  int nstage;             // attend pipeline depth (4..8)
  float scale_log2;
  long long total_rows;
  const void* q; long long q_sb, q_sg, q_sh;
  const void* k_cache; const void* v_cache;
  const long long* rows;
  void* out;
  float* part;
  unsigned* err;
};

template <typename KV_T, int HP>
__global__ void __launch_bounds__(kThreads, 1) attend_kernel(const AttendParams p) {
  using Cfg = AttendCfg<KV_T, HP>;
  extern __shared__ __align__(128) unsigned char dsm[];
  __shared__ float s_m[HP], s_l[HP];
  __shared__ float s_acc[HP * kHeadDim];
  cg::cluster_group cluster = cg::this_cluster();
  const int CS = (int)cluster.num_blocks();
  const int crank = (int)cluster.block_rank();
  const int seg = blockIdx.y;
  const int b = seg / p.G, g = seg - b * p.G;
  const int n_all = p.mode == 0 ? p.S : p.L;
  const int r0 = (int)(((long long)crank * n_all) / CS), r1 = (int)(((long long)(crank + 1) * n_all) / CS);
  RowSrc rs{nullptr, 0u};
  if (p.mode == 0) {
    uint32_t* s_arow = reinterpret_cast<uint32_t*>(dsm + Cfg::smem(p.nstage));
    for (int i = threadIdx.x; i < r1 - r0; i += kThreads)
      s_arow[i] = checked_row(p.rows[(size_t)seg * p.S + r0 + i], p.total_rows, p.err);
    __syncthreads();
    rs.list = s_arow;
  } else {
    rs.base = (uint32_t)((long long)seg * p.C + r0);
  }
  const float* s_q = stage_q<KV_T, HP>(dsm, p.nstage, reinterpret_cast<const KV_T*>(p.q) + b * p.q_sb + g * p.q_sg,
                                      p.q_sh, p.h);
  __syncthreads();
  attend_rows<KV_T, HP>(reinterpret_cast<const KV_T*>(p.k_cache), reinterpret_cast<const KV_T*>(p.v_cache), rs,
                        r1 - r0, s_q, p.scale_log2, dsm, p.nstage, s_m, s_l, s_acc);
  finish_output<KV_T, HP>(p.out ? reinterpret_cast<KV_T*>(p.out) + (size_t)seg * p.h * kHeadDim : nullptr,
                          p.part ? p.part + (size_t)seg * p.h * (kHeadDim + 2) : nullptr, p.h, s_m, s_l, s_acc);
}

}  // namespace al
