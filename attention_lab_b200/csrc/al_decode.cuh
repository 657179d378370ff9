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
  int canonical;
  int cpc;                // candidate columns per CTA
  int union_bytes;        // bytes of the keys / attend-engine union at the start of dynamic shared memory
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
template <typename IDX_T>
__device__ void compute_u(const DecodeParams& p, int b, int g, float* s_u, float* s_pre) {
  const int tid = threadIdx.x, seg = b * p.G + g;
  if (p.u_in) {
    if (tid < kMaxR) s_u[tid] = (tid < p.r) ? tof(reinterpret_cast<const IDX_T*>(p.u_in)[(size_t)seg * p.r + tid]) : 0.f;
    __syncthreads();
    return;
  }
  const IDX_T* qp = reinterpret_cast<const IDX_T*>(p.q_pre) + b * p.qp_sb + g * p.qp_sg;
  const int hd = p.h * kHeadDim;
  const IDX_T* wq = reinterpret_cast<const IDX_T*>(p.wq_t) + (size_t)g * hd * p.r;
  const int j = tid & 31, w = tid >> 5;
  float acc = 0.f;
  if (j < p.r) {
#pragma unroll 8
    for (int f = w; f < hd; f += kWarps) {
      const int hh = f / kHeadDim, dd = f % kHeadDim;
      acc = fmaf(tof(qp[hh * p.qp_sh + dd]), tof(wq[(size_t)f * p.r + j]), acc);
    }
  }
  s_pre[w * 32 + j] = acc;
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
  const int tid = threadIdx.x, j = tid >> 3, part = tid & 7, seg = b * p.G + g;
  const IDX_T* kn = reinterpret_cast<const IDX_T*>(p.k_new) + b * p.kn_sb + g * p.kn_sg;
  const IDX_T* wk = reinterpret_cast<const IDX_T*>(p.wk) + ((size_t)g * p.r + (j < p.r ? j : 0)) * kHeadDim;
  float acc = 0.f;
  if (j < p.r) {
#pragma unroll
    for (int e = part * 16; e < part * 16 + 16; ++e) acc = fmaf(tof(wk[e]), tof(kn[e]), acc);
  }
  acc += __shfl_xor_sync(0xffffffffu, acc, 1);
  acc += __shfl_xor_sync(0xffffffffu, acc, 2);
  acc += __shfl_xor_sync(0xffffffffu, acc, 4);
  if (j < p.r && part == 0)
    reinterpret_cast<IDX_T*>(p.zT)[((size_t)seg * p.r + j) * p.C + p.write_col] = fromf<IDX_T>(acc);
}

// Scores of candidate columns [c0, c1) -> order keys in s_keys[0, c1-c0) (and fp32 scores when requested).
template <typename IDX_T>
__device__ void scan_columns(const DecodeParams& p, int seg, int c0, int c1, const float* s_u, uint32_t* s_keys) {
  const IDX_T* zseg = reinterpret_cast<const IDX_T*>(p.zT) + (size_t)seg * p.r * p.C;
  float u[kMaxR];
#pragma unroll
  for (int j = 0; j < kMaxR; ++j) u[j] = s_u[j];
  float* so = p.scores_out ? p.scores_out + (size_t)seg * p.M - p.lo : nullptr;   // indexed by column
  if (p.zvec) {
    constexpr int VW = V16<IDX_T>::n;
    const int a0 = (c0 / VW) * VW;
    const int ngr = (c1 - a0 + VW - 1) / VW;
    for (int gi = threadIdx.x; gi < ngr; gi += kThreads) {
      const int col = a0 + gi * VW;
      const IDX_T* zc = zseg + col;
      float acc[VW];
#pragma unroll
      for (int e = 0; e < VW; ++e) acc[e] = 0.f;
#pragma unroll
      for (int jb = 0; jb < kMaxR; jb += 8) {
        uint4 v[8];
#pragma unroll
        for (int jj = 0; jj < 8; ++jj)
          v[jj] = (jb + jj < p.r) ? ldg_stream16(zc + (size_t)(jb + jj) * p.C) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
          float f[VW];
          unpack(v[jj], f, (const IDX_T*)nullptr);
#pragma unroll
          for (int e = 0; e < VW; ++e) acc[e] = fmaf(u[jb + jj], f[e], acc[e]);
        }
      }
#pragma unroll
      for (int e = 0; e < VW; ++e) {
        const int c = col + e;
        if (c >= c0 && c < c1) {
          s_keys[c - c0] = score_key(acc[e]);
          if (so) so[c] = acc[e];
        }
      }
    }
  } else {
    for (int c = c0 + threadIdx.x; c < c1; c += kThreads) {
      float a = 0.f;
      for (int j = 0; j < p.r; ++j) a = fmaf(s_u[j], tof(zseg[(size_t)j * p.C + c]), a);
      s_keys[c - c0] = score_key(a);
      if (so) so[c] = a;
    }
  }
}

template <typename KV_T, typename IDX_T, int HP>
__global__ void __launch_bounds__(kThreads, 1) sparse_step_kernel(const DecodeParams p) {
  extern __shared__ __align__(128) unsigned char dsm[];
  __shared__ float s_u[kMaxR];
  __shared__ float s_pre[kWarps * 32];
  __shared__ unsigned s_hist[2048];
  __shared__ unsigned s_slice[2048];
  __shared__ int s_sltot[kMaxCluster];
  __shared__ int s_cgt[kMaxCluster], s_ceq[kMaxCluster];
  __shared__ int s_piv[2];
  __shared__ int s_ws[kWarps];
  __shared__ int s_wgt[kWarps], s_weq[kWarps];
  __shared__ int s_fpre;
  __shared__ float s_m[HP], s_l[HP];
  __shared__ float s_acc[HP * kHeadDim];

  cg::cluster_group cluster = cg::this_cluster();
  const int CS = (int)cluster.num_blocks();
  const int crank = (int)cluster.block_rank();
  const int seg = blockIdx.y;
  const int b = seg / p.G, g = seg - b * p.G;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  uint32_t* s_keys = reinterpret_cast<uint32_t*>(dsm);
  uint32_t* s_arow = reinterpret_cast<uint32_t*>(dsm + p.union_bytes);

  // ---------------- prologue: z column (rank 0 of the cluster) and u ----------------
  if (p.k_new && crank == 0) write_z_column<IDX_T>(p, b, g);
  if (p.scan) compute_u<IDX_T>(p, b, g, s_u, s_pre);

  const int c0 = p.lo + crank * p.cpc;
  const int c1 = min(p.hi, c0 + p.cpc);
  const int nloc = max(0, c1 - c0);

  // ---------------- scan: candidate scores -> order keys in shared memory ----------------
  if (p.scan && nloc > 0) scan_columns<IDX_T>(p, seg, c0, c1, s_u, s_keys);
  __syncthreads();

  // ---------------- radix select of the k-th largest key over the cluster ----------------
  uint32_t tau = 0;
  int k_rem = 0;
  if (p.select_mode == 1) {
    uint32_t prefix = 0, pmask = 0;
    k_rem = p.k;
#pragma unroll 1
    for (int pass = 0; pass < 3; ++pass) {
      const int shift = pass == 0 ? 21 : (pass == 1 ? 10 : 0);
      const int NB = pass == 2 ? 1024 : 2048;
      for (int i = tid; i < NB; i += kThreads) s_hist[i] = 0u;
      __syncthreads();
      for (int i = tid; i < nloc; i += kThreads) {
        const uint32_t key = s_keys[i];
        if ((key & pmask) == prefix) atomicAdd(&s_hist[(key >> shift) & (NB - 1)], 1u);
      }
      cluster.sync();
      // reduce-scatter: this CTA sums bins [s0, s0 + SL) over the cluster
      const int SL = NB / CS, s0 = crank * SL;
      for (int i = tid; i < SL; i += kThreads) {
        unsigned v = 0;
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
      if (tid < CS) cluster.map_shared_rank(s_sltot, tid)[crank] = tot;
      cluster.sync();
      int cum = 0, ps = -1;
      for (int c = CS - 1; c >= 0; --c) {
        const int t2 = s_sltot[c];
        if (cum + t2 >= k_rem) { ps = c; break; }
        cum += t2;
      }
      if (ps == crank) {
        const int need = k_rem - cum;
        int above = tot - incl;
        for (int i = BPT - 1; i >= 0; --i) {
          const int bin = tid * BPT + i;
          if (bin < SL) {
            const int hv = (int)s_slice[bin];
            if (above < need && above + hv >= need) {
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
      cluster.sync();
      const int gt_add = s_piv[1];
      prefix |= (uint32_t)s_piv[0] << shift;
      pmask |= (uint32_t)(NB - 1) << shift;
      k_rem -= gt_add;
    }
    tau = prefix;   // the k-th largest key; k_rem of its copies (in position order) complete the top-k
  }

  // ---------------- compaction: chosen candidates in ascending position order ----------------
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
    const int WS = ((nloc + kWarps * 32 - 1) / (kWarps * 32)) * 32;
    const int wb = min(nloc, w * WS), we = min(nloc, wb + WS);
    int cgt = 0, ceq = 0;
    for (int base = wb; base < we; base += 32) {
      const int i = base + lane;
      const bool in = i < we;
      bool gt, eq;
      if (p.select_mode == 2) { gt = in; eq = false; }
      else { const uint32_t key = in ? s_keys[i] : 0u; gt = in && key > tau; eq = in && key == tau; }
      cgt += __popc(__ballot_sync(0xffffffffu, gt));
      ceq += __popc(__ballot_sync(0xffffffffu, eq));
    }
    if (lane == 0) { s_wgt[w] = cgt; s_weq[w] = ceq; }
    __syncthreads();
    if (tid < CS) {
      int tg = 0, te = 0;
      for (int i = 0; i < kWarps; ++i) { tg += s_wgt[i]; te += s_weq[i]; }
      cluster.map_shared_rank(s_cgt, tid)[crank] = tg;
      cluster.map_shared_rank(s_ceq, tid)[crank] = te;
    }
    cluster.sync();
    int eo = 0, so = 0;
    for (int c = 0; c < crank; ++c) {
      so += s_cgt[c] + min(max(k_rem - eo, 0), s_ceq[c]);
      eo += s_ceq[c];
    }
    const int sel_off = so;
    n_sel = s_cgt[crank] + min(max(k_rem - eo, 0), s_ceq[crank]);
    for (int i = 0; i < w; ++i) {
      so += s_wgt[i] + min(max(k_rem - eo, 0), s_weq[i]);
      eo += s_weq[i];
    }
    const int out_base = p.canonical ? s_fpre : F;
    long long* ro = p.rows_out ? p.rows_out + (size_t)seg * p.S + out_base : nullptr;
    const unsigned lt = (1u << lane) - 1u;
    for (int base = wb; base < we; base += 32) {
      const int i = base + lane;
      const bool in = i < we;
      bool gt, eq;
      if (p.select_mode == 2) { gt = in; eq = false; }
      else { const uint32_t key = in ? s_keys[i] : 0u; gt = in && key > tau; eq = in && key == tau; }
      const unsigned em = __ballot_sync(0xffffffffu, eq);
      const bool take = gt || (eq && (eo + __popc(em & lt)) < k_rem);
      const unsigned tm = __ballot_sync(0xffffffffu, take);
      if (take) {
        const int rank = so + __popc(tm & lt);
        const long long row = seg_off + (long long)(c0 - p.lo + i);
        if (ro) ro[rank] = row;
        s_arow[fshare + (rank - sel_off)] = checked_row(row, p.total_rows, p.err);
      }
      eo += __popc(em);
      so += __popc(tm);
    }
  }
  for (int i = tid; i < fshare; i += kThreads)
    s_arow[i] = checked_row(p.fixed_rows[(size_t)seg * F + fsh0 + i], p.total_rows, p.err);
  __syncthreads();
  if (p.rows_out && crank == 0 && w == 0) {
    // F into the row list: first (reference order), or around the candidates when canonical
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

  // ---------------- attend over this CTA's rows, then the cluster merge ----------------
  float q[HP][16];
  load_q<KV_T, HP>(reinterpret_cast<const KV_T*>(p.q) + b * p.q_sb + g * p.q_sg, p.q_sh, p.h, p.scale_log2, q);
  RowSrc rs{s_arow, 0u};
  attend_rows<KV_T, HP>(reinterpret_cast<const KV_T*>(p.k_cache), reinterpret_cast<const KV_T*>(p.v_cache), rs,
                        fshare + n_sel, q, dsm, s_m, s_l, s_acc);
  finish_output<KV_T, HP>(p.out ? reinterpret_cast<KV_T*>(p.out) + (size_t)seg * p.h * kHeadDim : nullptr,
                          p.part ? p.part + (size_t)seg * p.h * (kHeadDim + 2) : nullptr, p.h, s_m, s_l, s_acc);
}

// ------------------------------------------------------------------------------------------------ attend only
struct AttendParams {
  int B, G, h, C, S, L;
  int mode;               // 0: gathered rows [B,G,S] flat ids; 1: dense range [0, L) of each segment
  int rows_cap;
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
    uint32_t* s_arow = reinterpret_cast<uint32_t*>(dsm + Cfg::SMEM);
    for (int i = threadIdx.x; i < r1 - r0; i += kThreads)
      s_arow[i] = checked_row(p.rows[(size_t)seg * p.S + r0 + i], p.total_rows, p.err);
    __syncthreads();
    rs.list = s_arow;
  } else {
    rs.base = (uint32_t)((long long)seg * p.C + r0);
  }
  float q[HP][16];
  load_q<KV_T, HP>(reinterpret_cast<const KV_T*>(p.q) + b * p.q_sb + g * p.q_sg, p.q_sh, p.h, p.scale_log2, q);
  attend_rows<KV_T, HP>(reinterpret_cast<const KV_T*>(p.k_cache), reinterpret_cast<const KV_T*>(p.v_cache), rs,
                        r1 - r0, q, dsm, s_m, s_l, s_acc);
  finish_output<KV_T, HP>(p.out ? reinterpret_cast<KV_T*>(p.out) + (size_t)seg * p.h * kHeadDim : nullptr,
                          p.part ? p.part + (size_t)seg * p.h * (kHeadDim + 2) : nullptr, p.h, s_m, s_l, s_acc);
}

}  // namespace al
