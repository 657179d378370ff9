// Gather-free attention engine: one CTA attends its h query heads over a list of K/V rows read in place.
//
// Rows are flat ids into the flattened [B*G*C, d] cache (the reference's row-id convention, sparse.py:14-16).
// The engine streams the listed rows through shared memory with a 4-stage cp.async pipeline (16-byte chunks, a
// row is 16 threads x 16 B for bf16), in two sweeps per chunk of rows: a K sweep that scores every row for all h
// heads and keeps the scores in shared memory, then a V sweep that accumulates p * v with the chunk's exact maximum,
// so no per-row rescale is needed (one rescale per chunk of up to 1024 rows). Lane layout: 8 lanes per row, 16 dims
// per lane; the 8 lanes of a row reduce a dot product with 3 xor-shuffles. The result is the CTA's unnormalised
// partial (m, l, acc) per head in the log2 domain, merged across a thread-block cluster by `finish_output`.
#pragma once
#include "al_common.cuh"

namespace al {

template <typename KV_T, int HP>
struct AttendCfg {
  static constexpr int VE = V16<KV_T>::n;                 // elements per 16-byte chunk
  static constexpr int NCH = kHeadDim / VE;               // chunks per row
  static constexpr int NCL = NCH / 8;                     // chunks per lane
  static constexpr int ROWB = kHeadDim * (int)sizeof(KV_T);
  static constexpr int TR = (sizeof(KV_T) == 2) ? 64 : 32;  // rows per pipeline tile
  static constexpr int NSTAGE = 4;
  static constexpr int RPG = TR / 32;                     // rows per 8-lane group per tile
  static constexpr int CHUNK = 1024;                      // rows scored before their V sweep
  static constexpr int STAGE_BYTES = TR * ROWB;
  static constexpr int STAGES_BYTES = NSTAGE * STAGE_BYTES;
  static constexpr int RED_BYTES = kWarps * HP * kHeadDim * 4 + kWarps * HP * 4;
  static_assert(RED_BYTES <= STAGES_BYTES, "warp reduction buffer aliases the stage buffers");
  // shared memory of the engine: stage buffers | chunk scores | warp maxima
  static constexpr int SMEM = STAGES_BYTES + CHUNK * HP * 4 + kWarps * HP * 4;
};

// Row source: an explicit list in shared memory (0xffffffff marks a skipped row) or a contiguous range.
struct RowSrc {
  const uint32_t* list;
  uint32_t base;
  __device__ __forceinline__ uint32_t get(int i) const { return list ? list[i] : base + (uint32_t)i; }
};

template <typename Cfg>
__device__ __forceinline__ void issue_tile(const unsigned char* __restrict__ cache, RowSrc rows, int row0, int n,
                                           unsigned char* buf) {
  for (int ci = threadIdx.x; ci < Cfg::TR * Cfg::NCH; ci += kThreads) {
    const int rr = ci / Cfg::NCH, ch = ci % Cfg::NCH;
    const int row = row0 + rr;
    if (row < n) {
      const uint32_t id = rows.get(row);
      if (id != 0xffffffffu)
        cp_async16(buf + rr * Cfg::ROWB + ch * 16, cache + (size_t)id * Cfg::ROWB + ch * 16);
    }
  }
}

// Load this lane's 16 dims of row `rr` of a staged tile into floats.
template <typename KV_T, typename Cfg>
__device__ __forceinline__ void load_row(const unsigned char* buf, int rr, int li, float (&f)[16]) {
#pragma unroll
  for (int c = 0; c < Cfg::NCL; ++c) {
    const uint4 v = *reinterpret_cast<const uint4*>(buf + rr * Cfg::ROWB + (li + 8 * c) * 16);
    unpack(v, f + c * Cfg::VE, (const KV_T*)nullptr);
  }
}

// Dims held by lane li in slot e (0..15): chunk (li + 8*(e / VE)), element e % VE.
template <typename Cfg>
__device__ __forceinline__ int lane_dim(int li, int e) {
  return (li + 8 * (e / Cfg::VE)) * Cfg::VE + (e % Cfg::VE);
}

// Attend over rows[0, n_rows). q: this lane's dims, pre-multiplied by scale * log2(e). Writes the CTA partial
// (s_m[h], s_l[h], s_acc[h][128]) to shared memory; ends with a __syncthreads().
template <typename KV_T, int HP>
__device__ void attend_rows(const KV_T* __restrict__ Kf, const KV_T* __restrict__ Vf, RowSrc rows, int n_rows,
                            const float (&q)[HP][16], unsigned char* dsm, float* s_m, float* s_l, float* s_acc) {
  using Cfg = AttendCfg<KV_T, HP>;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5, lg = lane >> 3, li = lane & 7;
  unsigned char* stages = dsm;
  float* s_sc = reinterpret_cast<float*>(dsm + Cfg::STAGES_BYTES);
  float* s_wm = s_sc + Cfg::CHUNK * HP;
  const unsigned char* Kb = reinterpret_cast<const unsigned char*>(Kf);
  const unsigned char* Vb = reinterpret_cast<const unsigned char*>(Vf);

  float m_run[HP], l_run[HP], acc[HP][16];
#pragma unroll
  for (int hh = 0; hh < HP; ++hh) {
    m_run[hh] = -INFINITY;
    l_run[hh] = 0.f;
#pragma unroll
    for (int e = 0; e < 16; ++e) acc[hh][e] = 0.f;
  }

  for (int c0 = 0; c0 < n_rows; c0 += Cfg::CHUNK) {
    const int n = min(Cfg::CHUNK, n_rows - c0);
    RowSrc rs = rows;
    if (rs.list) rs.list += c0; else rs.base += (uint32_t)c0;
    const int ntiles = (n + Cfg::TR - 1) / Cfg::TR;
    float m_loc[HP];
#pragma unroll
    for (int hh = 0; hh < HP; ++hh) m_loc[hh] = -INFINITY;

    // ---------------- K sweep: scores of every row of the chunk ----------------
#pragma unroll
    for (int s = 0; s < Cfg::NSTAGE - 1; ++s) {
      if (s < ntiles) issue_tile<Cfg>(Kb, rs, s * Cfg::TR, n, stages + s * Cfg::STAGE_BYTES);
      cp_async_commit();
    }
    for (int t = 0; t < ntiles; ++t) {
      cp_async_wait<Cfg::NSTAGE - 2>();
      __syncthreads();
      const int tn = t + Cfg::NSTAGE - 1;
      if (tn < ntiles) issue_tile<Cfg>(Kb, rs, tn * Cfg::TR, n, stages + (tn % Cfg::NSTAGE) * Cfg::STAGE_BYTES);
      cp_async_commit();
      const unsigned char* buf = stages + (t % Cfg::NSTAGE) * Cfg::STAGE_BYTES;
#pragma unroll
      for (int i = 0; i < Cfg::RPG; ++i) {
        const int rr = (w * 4 + lg) * Cfg::RPG + i;
        const int row = t * Cfg::TR + rr;
        const bool valid = row < n && rs.get(row) != 0xffffffffu;
        float kf[16];
        if (valid) load_row<KV_T, Cfg>(buf, rr, li, kf);
        else {
#pragma unroll
          for (int e = 0; e < 16; ++e) kf[e] = 0.f;
        }
        float sc[HP];
#pragma unroll
        for (int hh = 0; hh < HP; ++hh) {
          float a = 0.f;
#pragma unroll
          for (int e = 0; e < 16; ++e) a = fmaf(q[hh][e], kf[e], a);
          sc[hh] = a;
        }
#pragma unroll
        for (int hh = 0; hh < HP; ++hh) {
          sc[hh] += __shfl_xor_sync(0xffffffffu, sc[hh], 1);
          sc[hh] += __shfl_xor_sync(0xffffffffu, sc[hh], 2);
          sc[hh] += __shfl_xor_sync(0xffffffffu, sc[hh], 4);
          if (!valid) sc[hh] = -INFINITY;
          m_loc[hh] = fmaxf(m_loc[hh], sc[hh]);
        }
        if (row < n && li < HP) {
          float v = sc[0];
#pragma unroll
          for (int hh = 1; hh < HP; ++hh) v = (li == hh) ? sc[hh] : v;
          s_sc[row * HP + li] = v;
        }
      }
    }
    cp_async_wait<0>();

    // chunk maximum per head, then one rescale of the running state
#pragma unroll
    for (int hh = 0; hh < HP; ++hh) {
      m_loc[hh] = fmaxf(m_loc[hh], __shfl_xor_sync(0xffffffffu, m_loc[hh], 8));
      m_loc[hh] = fmaxf(m_loc[hh], __shfl_xor_sync(0xffffffffu, m_loc[hh], 16));
    }
    if (lane < HP) {
      float v = m_loc[0];
#pragma unroll
      for (int hh = 1; hh < HP; ++hh) v = (lane == hh) ? m_loc[hh] : v;
      s_wm[w * HP + lane] = v;
    }
    __syncthreads();   // scores, warp maxima visible; every thread is done with the K tiles
#pragma unroll
    for (int hh = 0; hh < HP; ++hh) {
      float mc = -INFINITY;
#pragma unroll
      for (int i = 0; i < kWarps; ++i) mc = fmaxf(mc, s_wm[i * HP + hh]);
      const float mn = fmaxf(m_run[hh], mc);
      const float corr = (mn == -INFINITY) ? 1.f : exp2f(m_run[hh] - mn);
      m_run[hh] = mn;
      l_run[hh] *= corr;
#pragma unroll
      for (int e = 0; e < 16; ++e) acc[hh][e] *= corr;
    }

    // ---------------- V sweep: acc += exp2(s - m) * v ----------------
#pragma unroll
    for (int s = 0; s < Cfg::NSTAGE - 1; ++s) {
      if (s < ntiles) issue_tile<Cfg>(Vb, rs, s * Cfg::TR, n, stages + s * Cfg::STAGE_BYTES);
      cp_async_commit();
    }
    for (int t = 0; t < ntiles; ++t) {
      cp_async_wait<Cfg::NSTAGE - 2>();
      __syncthreads();
      const int tn = t + Cfg::NSTAGE - 1;
      if (tn < ntiles) issue_tile<Cfg>(Vb, rs, tn * Cfg::TR, n, stages + (tn % Cfg::NSTAGE) * Cfg::STAGE_BYTES);
      cp_async_commit();
      const unsigned char* buf = stages + (t % Cfg::NSTAGE) * Cfg::STAGE_BYTES;
#pragma unroll
      for (int i = 0; i < Cfg::RPG; ++i) {
        const int rr = (w * 4 + lg) * Cfg::RPG + i;
        const int row = t * Cfg::TR + rr;
        if (row < n && rs.get(row) != 0xffffffffu) {
          float p[HP];
#pragma unroll
          for (int hh = 0; hh < HP; ++hh) {
            const float sv = s_sc[row * HP + hh];
            p[hh] = (m_run[hh] == -INFINITY) ? 0.f : exp2f(sv - m_run[hh]);
            l_run[hh] += p[hh];
          }
          float vf[16];
          load_row<KV_T, Cfg>(buf, rr, li, vf);
#pragma unroll
          for (int hh = 0; hh < HP; ++hh)
#pragma unroll
            for (int e = 0; e < 16; ++e) acc[hh][e] = fmaf(p[hh], vf[e], acc[hh][e]);
        }
      }
    }
    cp_async_wait<0>();
    __syncthreads();   // V tiles consumed; the next chunk (or the reduction) may reuse the stage buffers
  }

  // ---------------- CTA reduction: 4 row groups per warp, then 8 warps ----------------
#pragma unroll
  for (int hh = 0; hh < HP; ++hh) {
    l_run[hh] += __shfl_xor_sync(0xffffffffu, l_run[hh], 8);
    l_run[hh] += __shfl_xor_sync(0xffffffffu, l_run[hh], 16);
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      acc[hh][e] += __shfl_xor_sync(0xffffffffu, acc[hh][e], 8);
      acc[hh][e] += __shfl_xor_sync(0xffffffffu, acc[hh][e], 16);
    }
  }
  float* red = reinterpret_cast<float*>(stages);           // [kWarps][HP][128]
  float* redl = red + kWarps * HP * kHeadDim;               // [kWarps][HP]
  if (lg == 0) {
#pragma unroll
    for (int hh = 0; hh < HP; ++hh)
#pragma unroll
      for (int e = 0; e < 16; ++e) red[(w * HP + hh) * kHeadDim + lane_dim<Cfg>(li, e)] = acc[hh][e];
    if (li < HP) {
      float v = l_run[0];
#pragma unroll
      for (int hh = 1; hh < HP; ++hh) v = (li == hh) ? l_run[hh] : v;
      redl[w * HP + li] = v;
    }
  }
  __syncthreads();
  for (int idx = tid; idx < HP * kHeadDim; idx += kThreads) {
    float a = 0.f;
#pragma unroll
    for (int i = 0; i < kWarps; ++i) a += red[i * HP * kHeadDim + idx];
    s_acc[idx] = a;
  }
  if (tid < HP) {
    float l = 0.f;
#pragma unroll
    for (int i = 0; i < kWarps; ++i) l += redl[i * HP + tid];
    s_l[tid] = l;
    float mv = m_run[0];
#pragma unroll
    for (int hh = 1; hh < HP; ++hh) mv = (tid == hh) ? m_run[hh] : mv;
    s_m[tid] = mv;
  }
  __syncthreads();
}

// Merge the cluster's partials and write out[h][128] (or, when `part` is given, the unnormalised partial of the
// whole cluster: part[h][130] = m (log2 domain), l, acc[128]). Every CTA of the cluster must call it.
template <typename KV_T, int HP>
__device__ void finish_output(KV_T* __restrict__ out, float* __restrict__ part, int h, const float* s_m,
                              const float* s_l, const float* s_acc) {
  cg::cluster_group cluster = cg::this_cluster();
  const int CS = (int)cluster.num_blocks();
  const int crank = (int)cluster.block_rank();
  if (CS > 1) cluster.sync();   // every CTA's partial is complete
  if (crank == 0) {
    for (int idx = threadIdx.x; idx < h * kHeadDim; idx += kThreads) {
      const int hh = idx / kHeadDim;
      float M = -INFINITY;
      for (int c = 0; c < CS; ++c) M = fmaxf(M, cluster.map_shared_rank(s_m, c)[hh]);
      float L = 0.f, A = 0.f;
      for (int c = 0; c < CS; ++c) {
        const float lc = cluster.map_shared_rank(s_l, c)[hh];
        if (lc > 0.f) {
          const float wgt = exp2f(cluster.map_shared_rank(s_m, c)[hh] - M);
          L = fmaf(wgt, lc, L);
          A = fmaf(wgt, cluster.map_shared_rank(s_acc, c)[idx], A);
        }
      }
      if (part) {
        part[hh * (kHeadDim + 2) + 2 + (idx % kHeadDim)] = A;
        if (idx % kHeadDim == 0) { part[hh * (kHeadDim + 2)] = M; part[hh * (kHeadDim + 2) + 1] = L; }
      } else {
        out[idx] = fromf<KV_T>(A / L);
      }
    }
  }
  if (CS > 1) cluster.sync();   // peers keep their shared memory alive until rank 0 has read it
}

// This lane's q dims (pre-scaled by scale*log2 e) for the heads of one (batch, group).
template <typename KV_T, int HP>
__device__ __forceinline__ void load_q(const KV_T* __restrict__ qb, long long sh, int h, float scale_log2,
                                       float (&q)[HP][16]) {
  using Cfg = AttendCfg<KV_T, HP>;
  const int li = threadIdx.x & 7;
#pragma unroll
  for (int hh = 0; hh < HP; ++hh)
#pragma unroll
    for (int e = 0; e < 16; ++e)
      q[hh][e] = (hh < h) ? tof(qb[hh * sh + lane_dim<Cfg>(li, e)]) * scale_log2 : 0.f;
}

}  // namespace al
