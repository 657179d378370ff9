// Gather-free attention engine: one CTA attends its h query heads over a list of K/V rows read in place.
//
// Rows are flat ids into the flattened [B*G*C, d] cache (the reference's row-id convention, sparse.py:14-16).
// The engine streams the listed rows through shared memory with a 3- to 5-stage cp.async pipeline of 32 KB tiles
// (128 bf16 or 64 fp32 rows; 16-byte chunks XOR-swizzled by row), one continuous tile stream across sweeps and
// chunks. Per chunk of up to CHUNK rows:
//   K tiles  - the scores of every (row, head): tensor cores for bf16 rows (mma.sync m16n8k16, the tile's rows as
//              A, the heads padded to 8 as B), CUDA cores for fp32 rows; stored head-major in shared memory;
//   chunk end - the chunk's exact per-head maximum rescales the running state once, then p = exp2(s - m) is
//              computed once per (row, head) (for bf16 rows rewritten in place as packed hi/lo bf16 fragments);
//   V tiles  - acc += p * v: tensor cores for bf16 rows (O^T = V^T P^T, two MMAs per step for p's hi and lo
//              halves), paired fp32 FMAs for fp32 rows.
// No per-row rescale is needed. The result is the CTA's unnormalised partial (m, l, acc) per head in the log2
// domain, merged across a thread-block cluster by `finish_output`.
#pragma once
#include "al_common.cuh"

namespace al {

template <typename KV_T, int HP>
struct AttendCfg {
  static constexpr int VE = V16<KV_T>::n;                 // elements per 16-byte chunk
  static constexpr int NCH = kHeadDim / VE;               // chunks per row (16 bf16, 32 fp32)
  static constexpr int NCL = NCH / 16;                    // chunks per lane in the V sweep (1 bf16, 2 fp32)
  static constexpr int ROWB = kHeadDim * (int)sizeof(KV_T);
  static constexpr int TR = (sizeof(KV_T) == 2) ? 128 : 64;  // rows per pipeline tile (32 KB)
  static constexpr int MIN_STAGES = 3;                    // pipeline depth is a runtime value in [3, MAX_STAGES]
  static constexpr int MAX_STAGES = 5;
  static constexpr int KPARTS = kThreads / TR;            // K sweep: threads per row (4 bf16, 8 fp32)
  static constexpr int KCH = NCH / KPARTS;                // K sweep: chunks per thread (4)
  static constexpr int LG = kThreads / 16;                // V sweep: 16-lane row groups per CTA
  static constexpr int RPG = TR / LG;                     // V sweep: rows per row group per tile
  static constexpr int CHUNK = 512;                       // rows scored before their V sweep
  // per-head stride of the chunk scores: CHUNK + 8 floats (= 8 mod 32 banks), so the V tile's probability fragments
  // (8 heads x 4 lanes of 8 bytes) and the K tile's score writes spread over the banks instead of sharing one
  static constexpr int SCS = CHUNK + 8;
  static constexpr int STAGE_BYTES = TR * ROWB;
  static constexpr int RED_BYTES = kWarps * HP * kHeadDim * 4;
  static_assert(RED_BYTES <= MIN_STAGES * STAGE_BYTES, "warp reduction buffer aliases the stage buffers");
  static_assert(RPG >= 1 && TR % LG == 0 && KCH * KPARTS == NCH && KPARTS * TR == kThreads, "tile shape");
  static_assert(CHUNK % TR == 0, "chunks hold whole tiles");
  static_assert(kWarps % 8 == 0 && TR % (16 * (kWarps / 8)) == 0, "V tile: 8 warps over the dims, the rest over rows");
  // shared memory of the engine with `stages` stages: stage buffers | chunk scores (then p) | warp maxima and sums |
  // fp32 rows only: K partial sums, q. (bf16 rows keep q in registers; it is staged in the last stage buffer.)
  static constexpr bool F32 = sizeof(KV_T) == 4;
  static constexpr int TAIL = SCS * HP * 4 + 2 * kWarps * HP * 4 + (F32 ? KPARTS * TR * HP * 4 + HP * kHeadDim * 4 : 0);
  static constexpr __host__ __device__ int smem(int stages) { return stages * STAGE_BYTES + TAIL; }
  static constexpr int SMEM = MIN_STAGES * STAGE_BYTES + TAIL;
  // a staged row holds its 16-byte chunks XOR-swizzled by the row index, so both sweeps read without bank conflicts
  static __device__ __forceinline__ int swz(int rr, int c) { return c ^ (rr & (NCH - 1)); }
};

// Row source: an explicit list in shared memory (0xffffffff marks a skipped row) or a contiguous range.
struct RowSrc {
  const uint32_t* list;
  uint32_t base;
  __device__ __forceinline__ uint32_t get(int i) const { return list ? list[i] : base + (uint32_t)i; }
};

// Every thread copies the same 16-byte chunk (tid % NCH) of rows tid / NCH + j * (kThreads / NCH) of the tile
// [row0, row0 + TR) into its swizzled place; rows at or beyond n, and skipped rows, are filled with zeros.
template <typename Cfg>
__device__ __forceinline__ void issue_tile(const unsigned char* __restrict__ cache, RowSrc rows, int row0, int n,
                                           unsigned char* buf) {
  constexpr int CPT = Cfg::TR * Cfg::NCH / kThreads;      // chunks per thread per tile
  constexpr int RSTEP = kThreads / Cfg::NCH;              // rows between a thread's chunks
  const int ch = threadIdx.x % Cfg::NCH, r0 = threadIdx.x / Cfg::NCH;
  const unsigned char* src = cache + ch * 16;
  // all row ids first (their shared-memory loads overlap), then the copies: a copy's memory clobber would otherwise
  // hold each next id load behind it
  uint32_t id[CPT];
#pragma unroll
  for (int j = 0; j < CPT; ++j) {
    const int row = row0 + r0 + j * RSTEP;
    id[j] = row < n ? rows.get(row) : 0xffffffffu;
  }
#pragma unroll
  for (int j = 0; j < CPT; ++j) {
    const int rr = r0 + j * RSTEP;
    unsigned char* dst = buf + rr * Cfg::ROWB + Cfg::swz(rr, ch) * 16;
    if (id[j] != 0xffffffffu) cp_async16(dst, src + (size_t)id[j] * Cfg::ROWB);
    else *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);   // rows not read hold zeros
  }
}

// 16-byte chunk (logical index c) of staged row rr as 4 float pairs (bf16: 8 dims; fp32: 4 dims in pairs 0-1).
template <typename KV_T, typename Cfg>
__device__ __forceinline__ void chunk2(const unsigned char* buf, int rr, int c, float2* f) {
  const uint4 v = *reinterpret_cast<const uint4*>(buf + rr * Cfg::ROWB + Cfg::swz(rr, c) * 16);
  if (sizeof(KV_T) == 2) {
    f[0] = make_float2(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xffff0000u));
    f[1] = make_float2(__uint_as_float(v.y << 16), __uint_as_float(v.y & 0xffff0000u));
    f[2] = make_float2(__uint_as_float(v.z << 16), __uint_as_float(v.z & 0xffff0000u));
    f[3] = make_float2(__uint_as_float(v.w << 16), __uint_as_float(v.w & 0xffff0000u));
  } else {
    f[0] = make_float2(__uint_as_float(v.x), __uint_as_float(v.y));
    f[1] = make_float2(__uint_as_float(v.z), __uint_as_float(v.w));
  }
}

// V sweep lane layout: lane li of a 16-lane row group owns chunk li (and li + 16 for fp32): 8 dims as 4 pairs.
template <typename KV_T, typename Cfg>
__device__ __forceinline__ void load_row2(const unsigned char* buf, int rr, int li, float2 (&f)[4]) {
#pragma unroll
  for (int c = 0; c < Cfg::NCL; ++c) chunk2<KV_T, Cfg>(buf, rr, li + 16 * c, f + 2 * c);
}

// Dim held by lane li of a row group in slot e (0..7) in the V sweep.
template <typename Cfg>
__device__ __forceinline__ int lane_dim(int li, int e) {
  return (li + 16 * (e / Cfg::VE)) * Cfg::VE + (e % Cfg::VE);
}

// Attend over rows[0, n_rows). s_q: the heads' q (pre-multiplied by scale * log2 e), HP x 128 floats in shared
// memory. Writes the CTA partial (s_m[HP], s_l[HP], s_acc[HP][128]); ends with a __syncthreads().
// K sweep: thread (part, rr) = (tid / TR, tid % TR) accumulates the dot products of staged row rr over chunks
// [part * KCH, (part + 1) * KCH) for every head (q reads are warp-uniform broadcasts); the KPARTS partial sums of a
// row are added through shared memory. V sweep: 16 lanes per row, 8 dims per lane. Products use Blackwell's paired
// fp32 FMA.
template <typename KV_T, int HP>
__device__ void attend_rows(const KV_T* __restrict__ Kf, const KV_T* __restrict__ Vf, RowSrc rows, int n_rows,
                            const float* s_q, float scale_log2, unsigned char* dsm, int nstage, float* s_m, float* s_l,
                            float* s_acc) {
  using Cfg = AttendCfg<KV_T, HP>;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5, li = lane & 15;
  const int grp = tid >> 4;                              // V sweep row group 0..LG-1
  const int krow = tid % Cfg::TR, kpart = tid / Cfg::TR; // K sweep row and dim part
  unsigned char* stages = dsm;
  float* s_sc = reinterpret_cast<float*>(dsm + nstage * Cfg::STAGE_BYTES);
  float* s_wm = s_sc + Cfg::SCS * HP;                    // [kWarps][HP] warp maxima
  float* s_wl = s_wm + kWarps * HP;                      // [kWarps][HP] warp sums of p
  float* s_kp = s_wl + kWarps * HP;                      // fp32 rows: [KPARTS][TR][HP] partial dot products
  const unsigned char* Kb = reinterpret_cast<const unsigned char*>(Kf);
  const unsigned char* Vb = reinterpret_cast<const unsigned char*>(Vf);

  float m_run[HP], l_run[HP];
  float2 acc[HP][4];                                    // fp32 rows: this lane's 8 dims per head
  // bf16 rows: O^T fragment (dims 16 (w & 7) + .., heads), as four independent accumulators (p's hi and lo parts
  // x even and odd row steps) so consecutive MMAs do not wait on each other; summed at the end
  float oc[4][4] = {};
#pragma unroll
  for (int hh = 0; hh < HP; ++hh) {
    m_run[hh] = -INFINITY;
    l_run[hh] = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[hh][i] = make_float2(0.f, 0.f);
  }

  // bf16 rows: q as the B operand of m16n8k16 (n = head, 8 heads with zeros beyond HP; k = 16 dims per step)
  uint32_t qb[8][2];
  if constexpr (sizeof(KV_T) == 2) {
    const int g = lane >> 2, t4 = lane & 3;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const float* qr = s_q + (g < HP ? g : 0) * kHeadDim + ks * 16 + 2 * t4;
      const float z = g < HP ? 1.f : 0.f;
      qb[ks][0] = pack_bf16x2(z * qr[0], z * qr[1]);
      qb[ks][1] = pack_bf16x2(z * qr[8], z * qr[9]);
    }
  }
  float mh[HP];                                         // per-head maxima of the scores this thread produced
#pragma unroll
  for (int hh = 0; hh < HP; ++hh) mh[hh] = -INFINITY;
  float mh2[2] = {-INFINITY, -INFINITY};                // bf16 rows: maxima of this lane's heads 2 t4, 2 t4 + 1

  // One continuous stream of tiles through the stage ring: for every chunk of up to CHUNK rows, its K tiles, then its
  // V tiles. Loads run nstage - 1 tiles ahead across sweep and chunk boundaries, so the ring never drains.
  struct Cursor {                                       // position in the tile stream
    int c0, n, nt, v, t;                                // chunk start, chunk rows, chunk tiles, V sweep?, tile
    __device__ __forceinline__ void start(int n_rows) { c0 = 0; n = min(Cfg::CHUNK, n_rows); nt = (n + Cfg::TR - 1) / Cfg::TR; v = 0; t = 0; }
    __device__ __forceinline__ bool valid() const { return nt > 0; }
    __device__ __forceinline__ void next(int n_rows) {
      if (++t < nt) return;
      t = 0;
      if (!v) { v = 1; return; }
      v = 0;
      c0 += Cfg::CHUNK;
      n = max(0, min(Cfg::CHUNK, n_rows - c0));
      nt = (n + Cfg::TR - 1) / Cfg::TR;
    }
  };
  auto chunk_rows = [&](const Cursor& cu) {
    RowSrc r = rows;
    if (r.list) r.list += cu.c0; else r.base += (uint32_t)cu.c0;
    return r;
  };
  Cursor ci, cc;                                        // issue cursor, consume cursor
  ci.start(n_rows);
  cc.start(n_rows);
  int sissue = 0, scons = 0;                            // stages of the next issue / consume
  for (int s = 0; s < nstage - 1; ++s) {
    if (ci.valid()) {
      issue_tile<Cfg>(ci.v ? Vb : Kb, chunk_rows(ci), ci.t * Cfg::TR, ci.n, stages + sissue * Cfg::STAGE_BYTES);
      ci.next(n_rows);
    }
    cp_async_commit();
    sissue = sissue + 1 == nstage ? 0 : sissue + 1;
  }
  while (cc.valid()) {
    cp_async_wait_dyn(nstage - 2);
    __syncthreads();                                    // this tile landed for everyone; the previous stage is free
    if (ci.valid()) {
      issue_tile<Cfg>(ci.v ? Vb : Kb, chunk_rows(ci), ci.t * Cfg::TR, ci.n, stages + sissue * Cfg::STAGE_BYTES);
      ci.next(n_rows);
    }
    cp_async_commit();
    sissue = sissue + 1 == nstage ? 0 : sissue + 1;
    const unsigned char* buf = stages + scons * Cfg::STAGE_BYTES;
    scons = scons + 1 == nstage ? 0 : scons + 1;
    const RowSrc rs = chunk_rows(cc);
    const int n = cc.n, t = cc.t;
    if (!cc.v) {
      // ---------------- K tile: scores of its rows ----------------
      if constexpr (sizeof(KV_T) == 2) {
        // tensor cores: warp w < TR/16 owns rows [16w, 16w + 16) of the tile; 8 steps of 16 dims
        if (w < Cfg::TR / 16) {
          const int lr = 16 * w + (lane & 15), lhi = lane >> 4;
          const uint32_t rowaddr = smem_addr(buf + lr * Cfg::ROWB);
          float ce[4] = {0.f, 0.f, 0.f, 0.f}, co[4] = {0.f, 0.f, 0.f, 0.f};   // even / odd dim steps
          uint32_t a[8][4];                               // every fragment first, then the MMAs
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)
            ldmatrix_x4(rowaddr + (uint32_t)(Cfg::swz(lr, 2 * ks + lhi) << 4), a[ks][0], a[ks][1], a[ks][2], a[ks][3]);
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)
            mma_bf16_16816((ks & 1) ? co : ce, a[ks][0], a[ks][1], a[ks][2], a[ks][3], qb[ks][0], qb[ks][1]);
          const float c[4] = {ce[0] + co[0], ce[1] + co[1], ce[2] + co[2], ce[3] + co[3]};
          // c0, c1: row 16w + g, heads 2 t4, 2 t4 + 1; c2, c3: row 16w + g + 8
          const int g = lane >> 2, t4 = lane & 3;
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            const int row = t * Cfg::TR + 16 * w + g + 8 * half;
            if (row < n) {
              const bool live = rs.get(row) != 0xffffffffu;
#pragma unroll
              for (int j = 0; j < 2; ++j) {
                const int head = 2 * t4 + j;
                if (head < HP) {
                  const float sc = live ? c[2 * half + j] * scale_log2 : -INFINITY;
                  s_sc[head * Cfg::SCS + row] = sc;
                  mh2[j] = fmaxf(mh2[j], sc);
                }
              }
            }
          }
        }
      } else {
        // CUDA cores (fp32 rows): thread (kpart, krow) sums its KCH chunks of row krow for every head; the KPARTS
        // partial sums of a row are added through shared memory
        {
          const int row = t * Cfg::TR + krow;
          const bool live = row < n && rs.get(row) != 0xffffffffu;
          float2 a[HP];
#pragma unroll
          for (int hh = 0; hh < HP; ++hh) a[hh] = make_float2(0.f, 0.f);
          if (live) {
#pragma unroll
            for (int j = 0; j < Cfg::KCH; ++j) {
              const int c = kpart * Cfg::KCH + j;
              float2 kf[4];
              chunk2<KV_T, Cfg>(buf, krow, c, kf);
#pragma unroll
              for (int hh = 0; hh < HP; ++hh) {
                const float4 q0 = *reinterpret_cast<const float4*>(s_q + hh * kHeadDim + c * Cfg::VE);
                a[hh] = __ffma2_rn(make_float2(q0.x, q0.y), kf[0], a[hh]);
                a[hh] = __ffma2_rn(make_float2(q0.z, q0.w), kf[1], a[hh]);
              }
            }
          }
          float* kp = s_kp + (kpart * Cfg::TR + krow) * HP;
#pragma unroll
          for (int hh = 0; hh < HP; ++hh) kp[hh] = a[hh].x + a[hh].y;
        }
        __syncthreads();                                // partial sums of the tile visible
        for (int i = tid; i < Cfg::TR * HP; i += kThreads) {
          const int rr = i / HP, head = i % HP;
          const int row = t * Cfg::TR + rr;
          if (row < n) {
            float sc = 0.f;
#pragma unroll
            for (int pp = 0; pp < Cfg::KPARTS; ++pp) sc += s_kp[pp * Cfg::TR * HP + i];
            sc = rs.get(row) == 0xffffffffu ? -INFINITY : sc * scale_log2;
            s_sc[head * Cfg::SCS + row] = sc;
#pragma unroll
            for (int hh = 0; hh < HP; ++hh) mh[hh] = (hh == head) ? fmaxf(mh[hh], sc) : mh[hh];
          }
        }
      }
      if (t == cc.nt - 1) {
        // ---------------- end of the chunk's K tiles: chunk maximum, one rescale, p = exp2(s - m) ----------------
        if (sizeof(KV_T) == 2) {
          const int t4 = lane & 3;
#pragma unroll
          for (int hh = 0; hh < HP; ++hh) mh[hh] = hh == 2 * t4 ? mh2[0] : (hh == 2 * t4 + 1 ? mh2[1] : mh[hh]);
          mh2[0] = mh2[1] = -INFINITY;
        }
#pragma unroll
        for (int hh = 0; hh < HP; ++hh)
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) mh[hh] = fmaxf(mh[hh], __shfl_xor_sync(0xffffffffu, mh[hh], o));
        if (lane == 0) {
#pragma unroll
          for (int hh = 0; hh < HP; ++hh) s_wm[w * HP + hh] = mh[hh];
        }
#pragma unroll
        for (int hh = 0; hh < HP; ++hh) mh[hh] = -INFINITY;
        __syncthreads();                                // scores + warp maxima visible
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
          if (sizeof(KV_T) == 2) {                      // O^T fragment columns are heads 2 t4 and 2 t4 + 1
            const int t4 = lane & 3;
#pragma unroll
            for (int a = 0; a < 4; ++a) {
              if (hh == 2 * t4) { oc[a][0] *= corr; oc[a][2] *= corr; }
              if (hh == 2 * t4 + 1) { oc[a][1] *= corr; oc[a][3] *= corr; }
            }
          }
        }
        // p for every (head, row) of the chunk's tiles (zero past the last row). bf16 rows: each pair of rows is
        // rewritten in place as the packed B fragment {bf16 hi(p0), hi(p1), lo(p0), lo(p1)}, lo = p - hi.
        float psum[HP];
        const int nr = cc.nt * Cfg::TR;                 // rows of the chunk's tiles
#pragma unroll
        for (int hh = 0; hh < HP; ++hh) {
          psum[hh] = 0.f;
          const float mv = m_run[hh];
          float* sh = s_sc + hh * Cfg::SCS;
          for (int rp = tid; rp < nr / 2; rp += kThreads) {
            const float2 sv = *reinterpret_cast<const float2*>(sh + 2 * rp);
            const float p0 = (2 * rp < n && mv != -INFINITY && sv.x != -INFINITY) ? exp2f(sv.x - mv) : 0.f;
            const float p1 = (2 * rp + 1 < n && mv != -INFINITY && sv.y != -INFINITY) ? exp2f(sv.y - mv) : 0.f;
            psum[hh] += p0 + p1;
            if (sizeof(KV_T) == 2) {
              const uint32_t hi = pack_bf16x2(p0, p1);
              const __nv_bfloat162 h2 = *reinterpret_cast<const __nv_bfloat162*>(&hi);
              const uint32_t lo = pack_bf16x2(p0 - __low2float(h2), p1 - __high2float(h2));
              *reinterpret_cast<uint2*>(sh + 2 * rp) = make_uint2(hi, lo);
            } else {
              *reinterpret_cast<float2*>(sh + 2 * rp) = make_float2(p0, p1);
            }
          }
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
        __syncthreads();                                // p and the sums visible
#pragma unroll
        for (int hh = 0; hh < HP; ++hh) {
          float sum = 0.f;
#pragma unroll
          for (int i = 0; i < kWarps; ++i) sum += s_wl[i * HP + hh];
          l_run[hh] += sum;
        }
      }
    } else {
      // ---------------- V tile: O += p * v ----------------
      if constexpr (sizeof(KV_T) == 2) {
        // tensor cores: O^T[dims x heads] += V^T[dims x rows] * P^T[rows x heads]. Warp w owns dims
        // [16 (w % 8), +16) and the tile's rows [RPW (w / 8), +RPW) in steps of 16. Each p is split into a bf16 high
        // part and a bf16 remainder (two MMAs), so p keeps about 16 mantissa bits; V is exact in bf16.
        constexpr int RPW = Cfg::TR / (kWarps / 8);       // rows per warp
        const int mb = w & 7, khalf = w >> 3;
        const int g = lane >> 2, t4 = lane & 3;
        const int vr_lane = (lane & 7) + ((lane >> 4) << 3), vc_lane = 2 * mb + ((lane >> 3) & 1);
        constexpr int NK = RPW / 16;                      // row steps of 16
        uint32_t a[NK][4];                                // every fragment of the tile first, then the MMAs
        uint2 f0[NK], f1[NK];
#pragma unroll
        for (int kk = 0; kk < NK; ++kk) {
          const int r16 = RPW * khalf + 16 * kk;          // first row of this step within the tile
          const int vr = r16 + vr_lane;
          ldmatrix_x4_trans(smem_addr(buf + vr * Cfg::ROWB + Cfg::swz(vr, vc_lane) * 16), a[kk][0], a[kk][1], a[kk][2],
                            a[kk][3]);
          // B fragment of head g (zero beyond HP): rows r16 + 2 t4 (+1) and + 8 (+9), packed by the p pass
          f0[kk] = make_uint2(0u, 0u);
          f1[kk] = make_uint2(0u, 0u);
          if (g < HP) {
            const float* ph = s_sc + g * Cfg::SCS + t * Cfg::TR + r16 + 2 * t4;
            f0[kk] = *reinterpret_cast<const uint2*>(ph);
            f1[kk] = *reinterpret_cast<const uint2*>(ph + 8);
          }
        }
#pragma unroll
        for (int kk = 0; kk < NK; ++kk) {
          mma_bf16_16816(oc[2 * (kk & 1)], a[kk][0], a[kk][1], a[kk][2], a[kk][3], f0[kk].x, f1[kk].x);
          mma_bf16_16816(oc[2 * (kk & 1) + 1], a[kk][0], a[kk][1], a[kk][2], a[kk][3], f0[kk].y, f1[kk].y);
        }
      } else {
        // CUDA cores (fp32 rows): 16 lanes per row, 8 dims per lane; the row group's rows are read first
        float2 vf[Cfg::RPG][4];
        float pr[Cfg::RPG][HP];
#pragma unroll
        for (int i = 0; i < Cfg::RPG; ++i) {
          const int rr = grp * Cfg::RPG + i;
          const int row = t * Cfg::TR + rr;
          const bool ok = row < n && rs.get(row) != 0xffffffffu;
          const int rrow = ok ? row : 0;
#pragma unroll
          for (int hh = 0; hh < HP; ++hh) pr[i][hh] = ok ? s_sc[hh * Cfg::SCS + rrow] : 0.f;
          load_row2<KV_T, Cfg>(buf, rr, li, vf[i]);
        }
#pragma unroll
        for (int i = 0; i < Cfg::RPG; ++i)
#pragma unroll
          for (int hh = 0; hh < HP; ++hh) {
            const float2 p2 = make_float2(pr[i][hh], pr[i][hh]);
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[hh][e] = __ffma2_rn(p2, vf[i][e], acc[hh][e]);
          }
      }
    }
    cc.next(n_rows);
  }
  cp_async_wait<0>();
  __syncthreads();   // every tile consumed; the reduction may reuse the stage buffers

  // ---------------- CTA reduction ----------------
  float* red = reinterpret_cast<float*>(stages);
  if constexpr (sizeof(KV_T) == 2) {
    // bf16 rows: red[row part][head][128] from the O^T fragments, then the row parts are added
    constexpr int KH = kWarps / 8;
    const int mb = w & 7, khalf = w >> 3, g = lane >> 2, t4 = lane & 3;
#pragma unroll
    for (int x = 0; x < 4; ++x) {
      const int head = 2 * t4 + (x & 1), dim = 16 * mb + g + 8 * (x >> 1);
      if (head < HP) red[(khalf * HP + head) * kHeadDim + dim] = (oc[0][x] + oc[2][x]) + (oc[1][x] + oc[3][x]);
    }
    __syncthreads();
    for (int idx = tid; idx < HP * kHeadDim; idx += kThreads) {
      float a = 0.f;
#pragma unroll
      for (int i = 0; i < KH; ++i) a += red[i * HP * kHeadDim + idx];
      s_acc[idx] = a;
    }
  } else {
    // fp32 rows: 2 row groups per warp, then the warps
#pragma unroll
    for (int hh = 0; hh < HP; ++hh)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        acc[hh][e].x += __shfl_xor_sync(0xffffffffu, acc[hh][e].x, 16);
        acc[hh][e].y += __shfl_xor_sync(0xffffffffu, acc[hh][e].y, 16);
      }
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

// Write the heads' q into the engine's shared q buffer (HP x 128 floats; heads >= h are zero; for bf16 rows the
// buffer is the last stage, which attend_rows reads before its first copy into that stage). Scores are scaled by
// scale*log2 e after the dot products. Must be followed by a __syncthreads() before attend_rows reads it.
template <typename KV_T, int HP>
__device__ __forceinline__ float* stage_q(unsigned char* dsm, int nstage, const KV_T* __restrict__ qb, long long sh,
                                          int h) {
  using Cfg = AttendCfg<KV_T, HP>;
  float* s_q = Cfg::F32 ? reinterpret_cast<float*>(dsm + nstage * Cfg::STAGE_BYTES) + Cfg::SCS * HP + 2 * kWarps * HP +
                              Cfg::KPARTS * Cfg::TR * HP
                        : reinterpret_cast<float*>(dsm + (nstage - 1) * Cfg::STAGE_BYTES);
  for (int i = threadIdx.x; i < HP * kHeadDim; i += kThreads) {
    const int hh = i / kHeadDim, d = i % kHeadDim;
    s_q[i] = hh < h ? tof(qb[hh * sh + d]) : 0.f;
  }
  return s_q;
}

}  // namespace al
