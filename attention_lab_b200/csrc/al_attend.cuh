// Gather-free attention engine: one CTA attends its h query heads over a list of K/V rows read in place.
//
// Rows are flat ids into the flattened [B*G*C, d] cache (the reference's row-id convention, sparse.py:14-16).
// The engine streams the listed rows through shared memory with a multi-stage cp.async pipeline (16-byte chunks, a
// bf16 row is 16 threads x 16 B; 4 to 8 stages of 64 rows, as shared memory allows), in three steps per chunk of up
// to 1024 rows. (One-dimensional bulk copies, one per 256-byte row, measured about 2.5x slower on B200: the copy
// engine's per-request cost dominates at this row size.)
//   K sweep  - 16 lanes per row, 8 dims per lane; the h partial dot products are reduced across the 16 lanes with a
//              transposed butterfly (5 shuffles for 4 heads) and the scores stored in shared memory;
//   p pass   - the chunk's exact per-head maximum rescales the running state once, then p = exp2(s - m) is computed
//              once per (row, head) in place and summed into l;
//   V sweep  - acc += p * v with the same 16-lane layout.
// No per-row rescale is needed. The result is the CTA's unnormalised partial (m, l, acc) per head in the log2
// domain, merged across a thread-block cluster by `finish_output`.
#pragma once
#include "al_common.cuh"

namespace al {

template <typename KV_T, int HP>
struct AttendCfg {
  static constexpr int VE = V16<KV_T>::n;                 // elements per 16-byte chunk
  static constexpr int NCH = kHeadDim / VE;               // chunks per row (16 bf16, 32 fp32)
  static constexpr int NCL = NCH / 16;                    // chunks per lane (1 bf16, 2 fp32)
  static constexpr int DPL = 8;                           // dims per lane
  static constexpr int ROWB = kHeadDim * (int)sizeof(KV_T);
  static constexpr int TR = (sizeof(KV_T) == 2) ? 64 : 32;  // rows per pipeline tile
  static constexpr int MIN_STAGES = 4;                    // pipeline depth is a runtime value in [4, MAX_STAGES]
  static constexpr int MAX_STAGES = 8;
  static constexpr int LG = kThreads / 16;                // 16-lane row groups per CTA
  static constexpr int RPG = TR / LG;                     // rows per row group per tile
  static constexpr int CHUNK = 1024;                      // rows scored before their V sweep
  static constexpr int STAGE_BYTES = TR * ROWB;
  static constexpr int RED_BYTES = kWarps * HP * kHeadDim * 4;
  static_assert(RED_BYTES <= MIN_STAGES * STAGE_BYTES, "warp reduction buffer aliases the stage buffers");
  static_assert(RPG >= 1 && TR % LG == 0, "tile rows must be a multiple of the row groups");
  // shared memory of the engine with `stages` stages: stage buffers | chunk scores (then p) | warp maxima and sums
  static constexpr int TAIL = CHUNK * HP * 4 + 2 * kWarps * HP * 4;
  static constexpr __host__ __device__ int smem(int stages) { return stages * STAGE_BYTES + TAIL; }
  static constexpr int SMEM = MIN_STAGES * STAGE_BYTES + TAIL;
};

// Row source: an explicit list in shared memory (0xffffffff marks a skipped row) or a contiguous range.
struct RowSrc {
  const uint32_t* list;
  uint32_t base;
  __device__ __forceinline__ uint32_t get(int i) const { return list ? list[i] : base + (uint32_t)i; }
};

// Every thread copies the same 16-byte chunk (tid % NCH) of rows tid / NCH + j * (kThreads / NCH) of the tile
// [row0, row0 + TR), for the rows below n that are not skipped.
template <typename Cfg>
__device__ __forceinline__ void issue_tile(const unsigned char* __restrict__ cache, RowSrc rows, int row0, int n,
                                           unsigned char* buf) {
  constexpr int CPT = Cfg::TR * Cfg::NCH / kThreads;      // chunks per thread per tile
  constexpr int RSTEP = kThreads / Cfg::NCH;              // rows between a thread's chunks
  const int ch = threadIdx.x % Cfg::NCH, r0 = threadIdx.x / Cfg::NCH;
#pragma unroll
  for (int j = 0; j < CPT; ++j) {
    const int rr = r0 + j * RSTEP;
    const int row = row0 + rr;
    if (row < n) {
      const uint32_t id = rows.get(row);
      if (id != 0xffffffffu)
        cp_async16(buf + rr * Cfg::ROWB + ch * 16, cache + (size_t)id * Cfg::ROWB + ch * 16);
    }
  }
}

// This lane's 8 dims of row `rr` of a staged tile (chunk li, and li + 16 for fp32) as 4 float pairs.
template <typename KV_T, typename Cfg>
__device__ __forceinline__ void load_row2(const unsigned char* buf, int rr, int li, float2 (&f)[4]) {
#pragma unroll
  for (int c = 0; c < Cfg::NCL; ++c) {
    const uint4 v = *reinterpret_cast<const uint4*>(buf + rr * Cfg::ROWB + (li + 16 * c) * 16);
    if (sizeof(KV_T) == 2) {
      f[0] = make_float2(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xffff0000u));
      f[1] = make_float2(__uint_as_float(v.y << 16), __uint_as_float(v.y & 0xffff0000u));
      f[2] = make_float2(__uint_as_float(v.z << 16), __uint_as_float(v.z & 0xffff0000u));
      f[3] = make_float2(__uint_as_float(v.w << 16), __uint_as_float(v.w & 0xffff0000u));
    } else {
      f[2 * c] = make_float2(__uint_as_float(v.x), __uint_as_float(v.y));
      f[2 * c + 1] = make_float2(__uint_as_float(v.z), __uint_as_float(v.w));
    }
  }
}

// Dim held by lane li in slot e (0..7).
template <typename Cfg>
__device__ __forceinline__ int lane_dim(int li, int e) {
  return (li + 16 * (e / Cfg::VE)) * Cfg::VE + (e % Cfg::VE);
}

// Head whose full 16-lane sum lane li holds after the transposed reduction (see reduce16).
template <int HP>
__device__ __forceinline__ int lane_head(int li) {
  if (HP == 4) return ((li >> 3) & 1) * 2 + ((li >> 2) & 1);
  if (HP == 2) return (li >> 3) & 1;
  return 0;
}

// Sum HP partial values over the 16 lanes of a row group. Lane li ends with the total of head lane_head<HP>(li).
template <int HP>
__device__ __forceinline__ float reduce16(const float (&v)[HP], int li) {
  if (HP == 4) {
    const bool b3 = (li >> 3) & 1, b2 = (li >> 2) & 1;
    float a0 = b3 ? v[2] : v[0], a1 = b3 ? v[3] : v[1];
    const float s0 = b3 ? v[0] : v[2], s1 = b3 ? v[1] : v[3];
    a0 += __shfl_xor_sync(0xffffffffu, s0, 8);
    a1 += __shfl_xor_sync(0xffffffffu, s1, 8);
    float b = b2 ? a1 : a0;
    b += __shfl_xor_sync(0xffffffffu, b2 ? a0 : a1, 4);
    b += __shfl_xor_sync(0xffffffffu, b, 2);
    b += __shfl_xor_sync(0xffffffffu, b, 1);
    return b;
  } else if (HP == 2) {
    const bool b3 = (li >> 3) & 1;
    float a = b3 ? v[1] : v[0];
    a += __shfl_xor_sync(0xffffffffu, b3 ? v[0] : v[1], 8);
    a += __shfl_xor_sync(0xffffffffu, a, 4);
    a += __shfl_xor_sync(0xffffffffu, a, 2);
    a += __shfl_xor_sync(0xffffffffu, a, 1);
    return a;
  } else {
    float a = v[0];
    a += __shfl_xor_sync(0xffffffffu, a, 8);
    a += __shfl_xor_sync(0xffffffffu, a, 4);
    a += __shfl_xor_sync(0xffffffffu, a, 2);
    a += __shfl_xor_sync(0xffffffffu, a, 1);
    return a;
  }
}

// Attend over rows[0, n_rows). q: this lane's 8 dims as 4 pairs, pre-multiplied by scale * log2(e). Writes the CTA
// partial (s_m[HP], s_l[HP], s_acc[HP][128]) to shared memory; ends with a __syncthreads(). Dot products and the
// p * v accumulation use Blackwell's paired fp32 FMA (two lanes of fp32 per instruction).
template <typename KV_T, int HP>
__device__ void attend_rows(const KV_T* __restrict__ Kf, const KV_T* __restrict__ Vf, RowSrc rows, int n_rows,
                            const float2 (&q)[HP][4], unsigned char* dsm, int nstage, float* s_m, float* s_l,
                            float* s_acc, unsigned* err) {
  using Cfg = AttendCfg<KV_T, HP>;
  (void)err;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5, li = lane & 15;
  const int grp = tid >> 4;                              // row group 0..LG-1
  unsigned char* stages = dsm;
  float* s_sc = reinterpret_cast<float*>(dsm + nstage * Cfg::STAGE_BYTES);
  float* s_wm = s_sc + Cfg::CHUNK * HP;                  // [kWarps][HP] warp maxima
  float* s_wl = s_wm + kWarps * HP;                      // [kWarps][HP] warp sums of p
  const unsigned char* Kb = reinterpret_cast<const unsigned char*>(Kf);
  const unsigned char* Vb = reinterpret_cast<const unsigned char*>(Vf);
  const int my_head = lane_head<HP>(li);
  const bool head_writer = (li & (16 / HP - 1)) == 0;   // one lane per head in each row group

  float m_run[HP], l_run[HP];
  float2 acc[HP][4];
#pragma unroll
  for (int hh = 0; hh < HP; ++hh) {
    m_run[hh] = -INFINITY;
    l_run[hh] = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[hh][i] = make_float2(0.f, 0.f);
  }

  for (int c0 = 0; c0 < n_rows; c0 += Cfg::CHUNK) {
    const int n = min(Cfg::CHUNK, n_rows - c0);
    RowSrc rs = rows;
    if (rs.list) rs.list += c0; else rs.base += (uint32_t)c0;
    const int ntiles = (n + Cfg::TR - 1) / Cfg::TR;
    float m_loc = -INFINITY;                            // max of this lane's head over its rows

    // ---------------- K sweep ----------------
    for (int s = 0; s < nstage - 1; ++s) {
      if (s < ntiles) issue_tile<Cfg>(Kb, rs, s * Cfg::TR, n, stages + s * Cfg::STAGE_BYTES);
      cp_async_commit();
    }
    int scur = 0, snext = nstage - 1;                   // stage of tile t, stage the next issue fills
    for (int t = 0; t < ntiles; ++t) {
      cp_async_wait_dyn(nstage - 2);
      __syncthreads();                                  // tile t landed for everyone; tile t-1's stage is free
      const int tn = t + nstage - 1;
      if (tn < ntiles) issue_tile<Cfg>(Kb, rs, tn * Cfg::TR, n, stages + snext * Cfg::STAGE_BYTES);
      cp_async_commit();
      const unsigned char* buf = stages + scur * Cfg::STAGE_BYTES;
      scur = scur + 1 == nstage ? 0 : scur + 1;
      snext = snext + 1 == nstage ? 0 : snext + 1;
#pragma unroll
      for (int i = 0; i < Cfg::RPG; ++i) {
        const int rr = grp * Cfg::RPG + i;
        const int row = t * Cfg::TR + rr;
        const bool valid = row < n && rs.get(row) != 0xffffffffu;
        float2 kf[4];
        if (valid) load_row2<KV_T, Cfg>(buf, rr, li, kf);
        else {
#pragma unroll
          for (int e = 0; e < 4; ++e) kf[e] = make_float2(0.f, 0.f);
        }
        float part[HP];
#pragma unroll
        for (int hh = 0; hh < HP; ++hh) {
          float2 a = __fmul2_rn(q[hh][0], kf[0]);
          a = __ffma2_rn(q[hh][1], kf[1], a);
          a = __ffma2_rn(q[hh][2], kf[2], a);
          a = __ffma2_rn(q[hh][3], kf[3], a);
          part[hh] = a.x + a.y;
        }
        float sc = reduce16<HP>(part, li);
        if (!valid) sc = -INFINITY;
        m_loc = fmaxf(m_loc, sc);
        if (row < n && head_writer) s_sc[row * HP + my_head] = sc;
      }
    }
    cp_async_wait<0>();

    // ---------------- chunk maximum, one rescale, p = exp2(s - m) in place ----------------
    m_loc = fmaxf(m_loc, __shfl_xor_sync(0xffffffffu, m_loc, 16));   // the other row group of the warp
    if (lane < 16 && head_writer) s_wm[w * HP + my_head] = m_loc;
    __syncthreads();                                    // scores + warp maxima visible; K tiles consumed
#pragma unroll
    for (int hh = 0; hh < HP; ++hh) {
      float mc = -INFINITY;
#pragma unroll
      for (int i = 0; i < kWarps; ++i) mc = fmaxf(mc, s_wm[i * HP + hh]);
      const float mn = fmaxf(m_run[hh], mc);
      const float corr = (mn == -INFINITY) ? 1.f : exp2f(m_run[hh] - mn);
      m_run[hh] = mn;
      l_run[hh] *= corr;
      const float2 c2 = make_float2(corr, corr);
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[hh][i] = __fmul2_rn(acc[hh][i], c2);
    }
    // V prologue first, so the loads overlap the exp pass
    for (int s = 0; s < nstage - 1; ++s) {
      if (s < ntiles) issue_tile<Cfg>(Vb, rs, s * Cfg::TR, n, stages + s * Cfg::STAGE_BYTES);
      cp_async_commit();
    }
    float psum[HP];
#pragma unroll
    for (int hh = 0; hh < HP; ++hh) psum[hh] = 0.f;
    for (int i = tid; i < n * HP; i += kThreads) {
      const int hh = i % HP;
      float mv = m_run[0];
#pragma unroll
      for (int x = 1; x < HP; ++x) mv = (hh == x) ? m_run[x] : mv;
      const float sv = s_sc[i];
      const float pv = (mv == -INFINITY || sv == -INFINITY) ? 0.f : exp2f(sv - mv);
      s_sc[i] = pv;
#pragma unroll
      for (int x = 0; x < HP; ++x) psum[x] += (hh == x) ? pv : 0.f;
    }
#pragma unroll
    for (int hh = 0; hh < HP; ++hh) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) psum[hh] += __shfl_xor_sync(0xffffffffu, psum[hh], o);
    }
    if (lane == 0) {
#pragma unroll
      for (int hh = 0; hh < HP; ++hh) s_wl[w * HP + hh] = psum[hh];
    }
    __syncthreads();                                    // p and the sums visible
#pragma unroll
    for (int hh = 0; hh < HP; ++hh) {
      float sum = 0.f;
#pragma unroll
      for (int i = 0; i < kWarps; ++i) sum += s_wl[i * HP + hh];
      l_run[hh] += sum;
    }

    // ---------------- V sweep: acc += p * v ----------------
    scur = 0;
    snext = nstage - 1;
    for (int t = 0; t < ntiles; ++t) {
      cp_async_wait_dyn(nstage - 2);
      __syncthreads();
      const int tn = t + nstage - 1;
      if (tn < ntiles) issue_tile<Cfg>(Vb, rs, tn * Cfg::TR, n, stages + snext * Cfg::STAGE_BYTES);
      cp_async_commit();
      const unsigned char* buf = stages + scur * Cfg::STAGE_BYTES;
      scur = scur + 1 == nstage ? 0 : scur + 1;
      snext = snext + 1 == nstage ? 0 : snext + 1;
#pragma unroll
      for (int i = 0; i < Cfg::RPG; ++i) {
        const int rr = grp * Cfg::RPG + i;
        const int row = t * Cfg::TR + rr;
        if (row < n && rs.get(row) != 0xffffffffu) {
          float p[HP];
          if (HP == 4) {
            const float4 p4 = *reinterpret_cast<const float4*>(s_sc + row * HP);
            p[0] = p4.x; p[1 % HP] = p4.y; p[2 % HP] = p4.z; p[3 % HP] = p4.w;
          } else {
#pragma unroll
            for (int hh = 0; hh < HP; ++hh) p[hh] = s_sc[row * HP + hh];
          }
          float2 vf[4];
          load_row2<KV_T, Cfg>(buf, rr, li, vf);
#pragma unroll
          for (int hh = 0; hh < HP; ++hh) {
            const float2 p2 = make_float2(p[hh], p[hh]);
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[hh][e] = __ffma2_rn(p2, vf[e], acc[hh][e]);
          }
        }
      }
    }
    cp_async_wait<0>();
    __syncthreads();   // V tiles and p consumed; the next chunk (or the reduction) may reuse the buffers
  }

  // ---------------- CTA reduction: 2 row groups per warp, then the warps ----------------
#pragma unroll
  for (int hh = 0; hh < HP; ++hh)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      acc[hh][e].x += __shfl_xor_sync(0xffffffffu, acc[hh][e].x, 16);
      acc[hh][e].y += __shfl_xor_sync(0xffffffffu, acc[hh][e].y, 16);
    }
  float* red = reinterpret_cast<float*>(stages);           // [kWarps][HP][128]
  if (lane < 16) {
#pragma unroll
    for (int hh = 0; hh < HP; ++hh)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        red[(w * HP + hh) * kHeadDim + lane_dim<Cfg>(li, 2 * e)] = acc[hh][e].x;
        red[(w * HP + hh) * kHeadDim + lane_dim<Cfg>(li, 2 * e + 1)] = acc[hh][e].y;
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
    float mv = m_run[0], lv = l_run[0];
#pragma unroll
    for (int hh = 1; hh < HP; ++hh) {
      mv = (tid == hh) ? m_run[hh] : mv;
      lv = (tid == hh) ? l_run[hh] : lv;
    }
    s_m[tid] = mv;
    s_l[tid] = lv;
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

// This lane's q dims (pre-scaled by scale*log2 e) for the heads of one (batch, group), as 4 pairs per head.
template <typename KV_T, int HP>
__device__ __forceinline__ void load_q(const KV_T* __restrict__ qb, long long sh, int h, float scale_log2,
                                       float2 (&q)[HP][4]) {
  using Cfg = AttendCfg<KV_T, HP>;
  const int li = threadIdx.x & 15;
#pragma unroll
  for (int hh = 0; hh < HP; ++hh)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float x = (hh < h) ? tof(qb[hh * sh + lane_dim<Cfg>(li, 2 * e)]) * scale_log2 : 0.f;
      const float y = (hh < h) ? tof(qb[hh * sh + lane_dim<Cfg>(li, 2 * e + 1)]) * scale_log2 : 0.f;
      q[hh][e] = make_float2(x, y);
    }
}

}  // namespace al
