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
// candidate columns. While it scans, each CTA counts its keys' top 12 bits and keeps only the keys that can still be
// in the top-k: a running lower bound of the k-th key's bin, read from the partial histogram, filters the keys
// appended to a short candidate list in shared memory (about k * (1 + ln(columns / round)) entries instead of one key
// per column). The radix histograms are reduce-scattered across the cluster through distributed shared memory, so
// the segment's exact k-th key is found without any global scratch; the chosen columns are marked in bitmaps and
// emitted in position order. Each CTA then attends over the candidates it selected plus a share of F, and the cluster
// merges the partial softmax states (log-sum-exp) into the output. Nothing is written to global memory except the
// z column, the output, and the optional row list and scores.
#pragma once
#include <cuda.h>
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
  int union_bytes;        // bytes of the selection / attend-engine union at the start of dynamic smem
  int bm_off, list_off;   // selection region: bitmaps and candidate list offsets (histogram at 0, slice at 16 KB)
  int nwp;                // words per selection bitmap
  int cap;                // candidate-list capacity per CTA (entries)
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
  unsigned long long* keys_out;                     // [B,G,kst] 64-bit keys of the chosen candidates, nullable
  long long key_pos;                                // position of column 0 in the keys (a shard's first position)
  int kst;                                          // keys_out entries per segment (>= k; the rest are zero)
  int skey_off;                                     // selection region: per-column keys (keys_out only)
  int tkeys;                                        // 1: resident-key scan (TMA tiles, keys in TMEM; select_mode 1)
  int ring_off, nring;                              // resident-key scan: ring offset in dynamic smem, stages
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
  static_assert(kThreads == 8 * kMaxR, "one 8-lane group per index row");
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

// Scores of candidate columns [c0, c1) -> order keys, handed to a sink. The scan runs in rounds of kThreads column
// groups; every lane of every warp calls sink.put<VW>(col, keys, scores, mask) once per round (warp-convergent: the
// sink may use warp collectives) with VW adjacent columns starting at `col` (bit e of `mask`: column col + e lies
// in [c0, c1)), then sink.round_end(round). Recomputing a column gives the same key bit for bit (same loads, same
// fused multiply-add order), so a sink may rescan. Vector path: each thread owns VW adjacent columns and streams all
// r rows of them with 16-byte loads; u is read from shared memory as broadcast float4s.
struct ZSrc {                                              // a segment's index columns zT[b, g] ([r, C])
  const void* z; int r, C, vec;                            // vec: 16-byte aligned rows
};

// Eight rows of a thread's VW columns: 16-byte loads, rows at or beyond r reread row r - 1 (u is zero there, and a
// non-finite z in row r - 1 already makes the true score non-finite).
template <typename IDX_T, bool FULLR>
__device__ __forceinline__ void load_rows8(uint4 (&v)[8], const IDX_T* zc, int j0, int r, int C) {
#pragma unroll
  for (int jj = 0; jj < 8; ++jj) v[jj] = ldg_stream16(zc + (size_t)(FULLR ? j0 + jj : min(j0 + jj, r - 1)) * C);
}

// acc += u[j0 + x] * z[x] for the eight rows held in v (rows in ascending order: the same FMA order on every path).
template <typename IDX_T>
__device__ __forceinline__ void fma_rows8(float2 (&acc2)[V16<IDX_T>::n / 2], const uint4 (&v)[8], const float* s_u,
                                          int j0) {
  constexpr int VW = V16<IDX_T>::n;
  const float4* u4 = reinterpret_cast<const float4*>(s_u + j0);
#pragma unroll
  for (int jq = 0; jq < 8; jq += 4) {
    const float4 uu = u4[jq / 4];
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

struct NoPre {
  __device__ __forceinline__ void operator()() const {}
};

// ------------------------------------------------------------------------------------ resident-key scan (TMA + TMEM)
// The segment's index columns [a0, c1) (a0 = c0 rounded down to 32) stream through shared memory as 2-D bulk-copy
// tiles of 32 rows x TW columns (16 KB: TW = 256 bf16 or 128 fp32 columns) in an NS-stage ring. A round is two tiles:
// threads 0-127 take the even tile, 128-255 the odd one; thread pp = tid % 128 of a half owns CPT adjacent columns
// (CPT = 2 bf16, 1 fp32: a 4-byte word per index row) and accumulates their scores over the 32 rows in ascending
// order with fp32 FMAs -- the arithmetic of scan_columns, so every key is bit-identical to the other scan paths.
// Every key goes to tensor memory (the CTA allocates 256 columns; the thread's lane, columns 128 half + CPT round + e),
// so the exact radix select afterwards re-reads all of them from TMEM instead of the index table: up to 32768 columns
// per CTA, no candidate list, no rescan. A column outside the CTA's candidates [c0, c1) stores key 0, which no score
// produces (keys below 0x00800000 would be NaN bit patterns, and NaN maps to 0xffffffff): every bin the select asks
// about is at least 7, so a key that passes its bin test is a valid candidate without further checks.
constexpr int kTileBytes = 16384;
constexpr int kMaxRing = 6;
constexpr uint32_t kTmemCols = 256;
constexpr int kTkeyMaxCols = 32768;            // columns [a0, c1) one CTA can hold in TMEM

template <typename IDX_T>
struct TKeyGeo {
  static constexpr int CPT = sizeof(IDX_T) == 2 ? 2 : 1;     // columns per thread per tile
  static constexpr int TW = 128 * CPT;                       // columns per tile
  static constexpr int ROWB = TW * (int)sizeof(IDX_T);       // bytes per tile row (512)
  int a0, c0, c1, ntiles, nrounds, nkeys, half, pp;
  uint32_t tlane;                                            // TMEM address of the thread's first key
  __device__ __forceinline__ TKeyGeo(int c0_, int c1_, uint32_t tbase) : c0(c0_), c1(c1_) {
    a0 = (c0 / 32) * 32;                                     // the selection bitmaps' first column: whole words
    ntiles = c1 > c0 ? (c1 - a0 + TW - 1) / TW : 0;
    nrounds = (ntiles + 1) / 2;
    nkeys = nrounds * CPT;
    half = threadIdx.x >> 7;
    pp = threadIdx.x & 127;
    tlane = tbase + ((uint32_t)(32 * ((threadIdx.x >> 5) & 3)) << 16) + 128u * (uint32_t)half;
  }
  // column of key i of this thread
  __device__ __forceinline__ int col(int i) const { return a0 + (2 * (i / CPT) + half) * TW + CPT * pp + i % CPT; }
  // col(i0 + e) - col(i0) for a chunk start i0 (a multiple of 8)
  static __device__ __forceinline__ int colstep(int e) { return (e / CPT) * 2 * TW + e % CPT; }
  // f(keys[8], i0) for each chunk of 8 of this thread's keys (key i0 + e in keys[e]; entries past the thread's keys
  // read as 0, like a column outside the candidates); every thread of the CTA calls it (warp-collective loads)
  template <typename F>
  __device__ __forceinline__ void for_each_chunk(F&& f) const {
    for (int q = 0; q * 8 < nkeys; ++q) {
      uint32_t r[8];
      tmem_ld8(tlane + 8u * q, r);
      tmem_wait_ld();
      if (8 * q + 8 > nkeys) {
#pragma unroll
        for (int e = 0; e < 8; ++e) r[e] = 8 * q + e < nkeys ? r[e] : 0u;
      }
      f(r, 8 * q);
    }
  }
};

// Issue tile t of the CTA's columns into ring stage t % nring.
template <typename IDX_T>
__device__ __forceinline__ void tkey_issue(const TKeyGeo<IDX_T>& g, const void* map, unsigned char* ring,
                                           uint64_t* full, int nring, int seg_row, int t) {
  const int s = t % nring;
  mbar_arrive_expect_tx(&full[s], kTileBytes);
  tma_load_2d(ring + s * kTileBytes, map, g.a0 + t * g.TW, seg_row, &full[s]);
}

// Named barrier of one half of the CTA (threads 128 h .. 128 h + 127; ids 1 and 2).
__device__ __forceinline__ void half_sync(int half) {
  asm volatile("bar.sync %0, 128;\n" ::"r"(1 + half) : "memory");
}

// The scan proper (after tkey_issue of the first min(nring, ntiles) tiles and with u in s_u): scores -> keys -> 12-bit
// histogram (s_hp: 2048 words, bins 2i and 2i+1 in the low and high 16 bits of word i; a CTA has at most 32768 keys,
// so no count overflows its half), optional fp32 scores (so, indexed by column), keys to TMEM. The two halves run
// independently: nring is even, so half h only ever waits on and refills the stages of its own tiles (t = h mod 2),
// and its leader thread re-arms a stage as soon as the half's 128 threads have read it. Returns false if a bounded
// wait gave up.
template <typename IDX_T>
__device__ __noinline__ bool tkey_scan(const TKeyGeo<IDX_T> g, const void* map, unsigned char* ring, uint64_t* full, int nring,
                          int seg_row, const float* s_u, unsigned* s_hp, float* so) {
  using Geo = TKeyGeo<IDX_T>;
  const float4* u4 = reinterpret_cast<const float4*>(s_u);   // broadcast reads, four rows at a time
  bool ok = true;
  const auto count = [&](uint32_t key) {
    const uint32_t bin = key >> 20;
    atomicAdd(&s_hp[bin >> 1], (bin & 1u) ? 0x10000u : 1u);
  };
#pragma unroll 1
  for (int ri = 0; ri < g.nrounds; ++ri) {
    const int t = 2 * ri + g.half;
    if (t < g.ntiles) {                                     // uniform over each half (four whole warps)
      const int s = t % nring;
      ok = mbar_wait(&full[s], (unsigned)((t / nring) & 1)) && ok;
      const unsigned char* tile = ring + s * kTileBytes + g.pp * 4;
      if (Geo::CPT == 2) {
        float2 acc = make_float2(0.f, 0.f);
#pragma unroll
        for (int jq = 0; jq < kMaxR; jq += 4) {
          const float4 uq = u4[jq / 4];
          const float uj[4] = {uq.x, uq.y, uq.z, uq.w};
#pragma unroll
          for (int x = 0; x < 4; ++x) {
            const uint32_t wv = *reinterpret_cast<const uint32_t*>(tile + (jq + x) * Geo::ROWB);
            acc = __ffma2_rn(make_float2(uj[x], uj[x]), make_float2(__uint_as_float(wv << 16),
                                                                     __uint_as_float(wv & 0xffff0000u)), acc);
          }
        }
        const int c = g.a0 + t * Geo::TW + 2 * g.pp;
        const bool in0 = c >= g.c0 && c < g.c1, in1 = c + 1 >= g.c0 && c + 1 < g.c1;
        const uint32_t k0 = in0 ? score_key(acc.x) : 0u, k1 = in1 ? score_key(acc.y) : 0u;
        if (in0) { count(k0); if (so) so[c] = acc.x; }
        if (in1) { count(k1); if (so) so[c + 1] = acc.y; }
        tmem_st2(g.tlane + 2u * ri, k0, k1);
      } else {
        float acc = 0.f;
#pragma unroll
        for (int jq = 0; jq < kMaxR; jq += 4) {
          const float4 uq = u4[jq / 4];
          const float uj[4] = {uq.x, uq.y, uq.z, uq.w};
#pragma unroll
          for (int x = 0; x < 4; ++x)
            acc = fmaf(uj[x], __uint_as_float(*reinterpret_cast<const uint32_t*>(tile + (jq + x) * Geo::ROWB)), acc);
        }
        const int c = g.a0 + t * Geo::TW + g.pp;
        const bool in0 = c >= g.c0 && c < g.c1;
        const uint32_t k0 = in0 ? score_key(acc) : 0u;
        if (in0) { count(k0); if (so) so[c] = acc; }
        tmem_st1(g.tlane + (uint32_t)ri, k0);
      }
    } else {                                                // no tile for this half in the last round: keys 0
      if (Geo::CPT == 2) tmem_st2(g.tlane + 2u * ri, 0u, 0u);
      else tmem_st1(g.tlane + (uint32_t)ri, 0u);
    }
    half_sync(g.half);                                      // this half's tile t is consumed
    if (g.pp == 0 && t + nring < g.ntiles) tkey_issue(g, map, ring, full, nring, seg_row, t + nring);
  }
  return ok;
}

// `pre` runs once, after the first two batches of loads are in flight and before u is first read (the fused kernel
// computes u there, so its latency hides under the loads); it must be called by every thread of the CTA.
template <typename IDX_T, bool FULLR, typename Sink, typename Pre>
__device__ __forceinline__ void scan_columns_impl(const ZSrc zs, int c0, int c1, const float* s_u, Sink sink, Pre pre) {
  const IDX_T* zseg = reinterpret_cast<const IDX_T*>(zs.z);
  const int r = FULLR ? kMaxR : zs.r, C = zs.C;
  if (zs.vec) {
    // Software pipeline over 8-row batches (4 per round): two batches are always in flight, and each batch is
    // multiplied while the next one loads; the next round's first two batches load during this round's last two.
    // A thread past the end of the columns rereads column a0 and its results are masked.
    constexpr int VW = V16<IDX_T>::n;
    static_assert(kMaxR == 32, "four 8-row batches per round");
    const int a0 = (c0 / VW) * VW;
    const int ngr = (c1 - a0 + VW - 1) / VW;
    const int nrounds = (ngr + kThreads - 1) / kThreads;
    uint4 va[8], vb[8];
    int gi = threadIdx.x;
    const IDX_T* zc = zseg + (gi < ngr ? a0 + gi * VW : a0);
    if (nrounds > 0) {
      load_rows8<IDX_T, FULLR>(va, zc, 0, r, C);
      load_rows8<IDX_T, FULLR>(vb, zc, 8, r, C);
    }
    pre();
#pragma unroll 1
    for (int round = 0; round < nrounds; ++round, gi += kThreads) {
      const bool in = gi < ngr;
      const int col = a0 + gi * VW;
      const int gn = gi + kThreads;
      const IDX_T* zn = zseg + (gn < ngr ? a0 + gn * VW : a0);
      const bool more = round + 1 < nrounds;
      float2 acc2[VW / 2];
#pragma unroll
      for (int e = 0; e < VW / 2; ++e) acc2[e] = make_float2(0.f, 0.f);
      fma_rows8<IDX_T>(acc2, va, s_u, 0);
      load_rows8<IDX_T, FULLR>(va, zc, 16, r, C);
      fma_rows8<IDX_T>(acc2, vb, s_u, 8);
      load_rows8<IDX_T, FULLR>(vb, zc, 24, r, C);
      fma_rows8<IDX_T>(acc2, va, s_u, 16);
      if (more) load_rows8<IDX_T, FULLR>(va, zn, 0, r, C);
      fma_rows8<IDX_T>(acc2, vb, s_u, 24);
      if (more) load_rows8<IDX_T, FULLR>(vb, zn, 8, r, C);
      zc = zn;
      float acc[VW];
      uint32_t kk[VW];
      unsigned vm = 0;
#pragma unroll
      for (int e = 0; e < VW / 2; ++e) { acc[2 * e] = acc2[e].x; acc[2 * e + 1] = acc2[e].y; }
#pragma unroll
      for (int e = 0; e < VW; ++e) {
        kk[e] = score_key(acc[e]);
        vm |= (in && col + e >= c0 && col + e < c1) ? (1u << e) : 0u;
      }
      sink.template put<VW>(col, kk, acc, vm);
      sink.round_end(round);
    }
  } else {
    pre();
#pragma unroll 1
    for (int cb = c0, round = 0; cb < c1; cb += kThreads, ++round) {
      const int c = cb + threadIdx.x;
      const bool in = c < c1;
      float a = 0.f;
      if (in)
        for (int j = 0; j < r; ++j) a = fmaf(s_u[j], tof(zseg[(size_t)j * C + c]), a);
      const uint32_t key = score_key(a);
      sink.template put<1>(c, &key, &a, in ? 1u : 0u);
      sink.round_end(round);
    }
  }
}

// r == 32 (every row real) takes a version without the row clamp.
template <typename IDX_T, typename Sink, typename Pre = NoPre>
__device__ __forceinline__ void scan_columns(const ZSrc zs, int c0, int c1, const float* s_u, const Sink& sink,
                                             const Pre& pre = Pre()) {
  if (zs.r == kMaxR) scan_columns_impl<IDX_T, true>(zs, c0, c1, s_u, sink, pre);
  else scan_columns_impl<IDX_T, false>(zs, c0, c1, s_u, sink, pre);
}

// Selection state of the fused kernel at fixed shared addresses (no registers needed to reach it): the dynamic
// region starts with the 4096-bin histogram; the candidate count and the filter threshold are static.
extern __shared__ __align__(128) unsigned char g_dsm[];
__shared__ unsigned g_list_count, g_list_thr;

__device__ __forceinline__ uint4 lds_volatile_u4(const void* p) {
  uint4 r;
  asm volatile("ld.volatile.shared.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(smem_addr(p)));
  return r;
}

// One warp raises the CTA's filter threshold *thr (a bin of the 12-bit key histogram) to the highest bin b whose
// suffix count sum(hist[b..4095]) reaches k. The histogram is read while other warps still add to it: the counts
// read are never above the final ones, so the result never exceeds the final bin of the k-th largest key (of the CTA,
// and so of the whole cluster), and every key of a top-k bin passes the filter. The threshold only increases.
__device__ void raise_threshold(const unsigned* hist, unsigned* thr, int k) {
  const int lane = threadIdx.x & 31;
  int t0 = 0;
  if (lane == 0) t0 = (int)*reinterpret_cast<volatile unsigned*>(thr);
  t0 = __shfl_sync(0xffffffffu, t0, 0);
  unsigned cum = 0;
  // four 128-bin blocks per step, their loads and sums independent; block i of a step covers bins
  // [top - 128 i - 127, top - 128 i], lane L holding its 4 bins top - 128 i - 4 L - 3 .. top - 128 i - 4 L
  for (int top = 4095; top >= t0; top -= 512) {
    uint4 v[4];
    unsigned ls[4], blk[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = lds_volatile_u4(hist + (top - 128 * i - 4 * lane - 3));
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      ls[i] = v[i].x + v[i].y + v[i].z + v[i].w;
      blk[i] = __reduce_add_sync(0xffffffffu, ls[i]);
    }
    int ib = -1;                                             // the block where the count from the top reaches k
    unsigned before = cum;
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (ib < 0) {
        if (before + blk[i] >= (unsigned)k) ib = i;
        else before += blk[i];
      }
    if (ib >= 0) {
      uint4 vv = v[0];
      unsigned lss = ls[0];
#pragma unroll
      for (int i = 1; i < 4; ++i)
        if (i == ib) { vv = v[i]; lss = ls[i]; }
      const int lo = top - 128 * ib - 4 * lane - 3;
      unsigned incl = lss;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
      }
      const int L = __ffs(__ballot_sync(0xffffffffu, before + incl >= (unsigned)k)) - 1;
      int bn = lo;
      unsigned c = before + incl - lss;
      if ((c += vv.w) >= (unsigned)k) bn = lo + 3;
      else if ((c += vv.z) >= (unsigned)k) bn = lo + 2;
      else if ((c += vv.y) >= (unsigned)k) bn = lo + 1;
      bn = __shfl_sync(0xffffffffu, bn, L);
      if (lane == 0 && bn > t0) *reinterpret_cast<volatile unsigned*>(thr) = (unsigned)bn;
      return;
    }
    cum = before;
  }
}

// First pass of the radix select: every valid key's top 12 bits are counted, and the keys whose bin is at or above
// the running threshold are appended to the CTA's candidate list (keys[cap] then columns - kb [cap]; warp-aggregated:
// one shared atomic per warp and round). The list keeps counting past its capacity so that an overflow is visible.
template <bool SCORES>
struct SinkFirst {
  float* so; int list_off, cap, k, kb;
  template <int VW>
  __device__ __forceinline__ void put(int col, const uint32_t* kk, const float* sc, unsigned vm) {
    unsigned* hist = reinterpret_cast<unsigned*>(g_dsm);
    const unsigned t = *reinterpret_cast<volatile unsigned*>(&g_list_thr);
    unsigned pm = 0;
#pragma unroll
    for (int e = 0; e < VW; ++e)
      if ((vm >> e) & 1u) {
        atomicAdd(&hist[kk[e] >> 20], 1u);
        if (SCORES) so[col + e] = sc[e];
        if ((kk[e] >> 20) >= t) pm |= 1u << e;
      }
    if (__any_sync(0xffffffffu, pm != 0u)) {
      // slots ordered by (e, lane): the lanes' stores of one e are contiguous (no bank conflicts)
      const unsigned lt = (1u << (threadIdx.x & 31)) - 1u;
      unsigned bal[VW];
      unsigned tot = 0;
#pragma unroll
      for (int e = 0; e < VW; ++e) {
        bal[e] = __ballot_sync(0xffffffffu, (pm >> e) & 1u);
        tot += __popc(bal[e]);
      }
      unsigned base = 0;
      if ((threadIdx.x & 31) == 0) base = atomicAdd(&g_list_count, tot);
      base = __shfl_sync(0xffffffffu, base, 0);
      uint32_t* lkey = reinterpret_cast<uint32_t*>(g_dsm + list_off);
      uint32_t* lcol = lkey + cap;
#pragma unroll
      for (int e = 0; e < VW; ++e) {
        const unsigned o = base + __popc(bal[e] & lt);
        if (((pm >> e) & 1u) && o < (unsigned)cap) {
          lkey[o] = kk[e];
          lcol[o] = (uint32_t)(col + e - kb);
        }
        base += __popc(bal[e]);
      }
    }
  }
  // every warp tightens the threshold after the first round (its keys were all appended), then one warp per round
  __device__ __forceinline__ void round_end(int round) {
    if (round == 0 || (int)(threadIdx.x >> 5) == round % kWarps)
      raise_threshold(reinterpret_cast<const unsigned*>(g_dsm), &g_list_thr, k);
  }
};

// Rescan sink, used when some CTA's candidate list overflowed: either a 10-bit digit histogram of the keys under a
// prefix (marks == false), or the selection marks (bitmaps over columns - kb of the keys above and equal to tau).
struct SinkRescan {
  bool marks;
  unsigned* hist; uint32_t prefix, pmask; int shift;
  uint32_t* gt; uint32_t* eq; uint32_t tau; int kb;
  uint32_t* skey;                                            // per-column keys of the marked columns, nullable
  template <int VW>
  __device__ __forceinline__ void put(int col, const uint32_t* kk, const float*, unsigned vm) {
    if (!marks) {
#pragma unroll
      for (int e = 0; e < VW; ++e)
        if (((vm >> e) & 1u) && (kk[e] & pmask) == prefix) atomicAdd(&hist[(kk[e] >> shift) & 1023u], 1u);
      return;
    }
    unsigned gm = 0, em = 0;
#pragma unroll
    for (int e = 0; e < VW; ++e)
      if ((vm >> e) & 1u) {
        gm |= (kk[e] > tau) ? (1u << e) : 0u;
        em |= (kk[e] == tau) ? (1u << e) : 0u;
      }
    const int rel = col - kb;                                // a multiple of VW: the VW bits share one word
    if (gm) atomicOr(&gt[rel >> 5], gm << (rel & 31));
    if (em) atomicOr(&eq[rel >> 5], em << (rel & 31));
    if (skey) {
#pragma unroll
      for (int e = 0; e < VW; ++e)
        if (((gm | em) >> e) & 1u) skey[rel + e] = kk[e];
    }
  }
  __device__ __forceinline__ void round_end(int) {}
};

// Every candidate chosen (k == M) but the keys requested: store every valid column's key.
struct SinkKeys {
  uint32_t* skey; int kb; float* so;
  template <int VW>
  __device__ __forceinline__ void put(int col, const uint32_t* kk, const float* sc, unsigned vm) {
#pragma unroll
    for (int e = 0; e < VW; ++e)
      if ((vm >> e) & 1u) {
        skey[col + e - kb] = kk[e];
        if (so) so[col + e] = sc[e];
      }
  }
  __device__ __forceinline__ void round_end(int) {}
};

// 64-bit candidate key: the score's order key above the inverted position, so a larger key ranks first under
// (score desc, position asc) and no two positions tie.
__device__ __forceinline__ unsigned long long pack_key64(uint32_t key, long long pos) {
  return ((unsigned long long)key << 32) | (unsigned long long)(0xffffffffu - (uint32_t)pos);
}

// Scores only (no top-k): write the fp32 scores.
struct SinkScores {
  float* so;
  template <int VW>
  __device__ __forceinline__ void put(int col, const uint32_t*, const float* sc, unsigned vm) {
#pragma unroll
    for (int e = 0; e < VW; ++e)
      if ((vm >> e) & 1u) so[col + e] = sc[e];
  }
  __device__ __forceinline__ void round_end(int) {}
};

// One warp: the bin of a 4096-bin histogram holding the need-th largest element counted from the top bin, the
// number of elements above that bin, and the bin's own count.
__device__ void warp_pivot4096(const unsigned* hist, int need, int& bin_out, int& above_out, int& count_out) {
  const int lane = threadIdx.x & 31;
  unsigned cum = 0;
  bin_out = 0; above_out = 0; count_out = 0;
  for (int top = 4095; top >= 0; top -= 128) {
    const int lo = top - 4 * lane - 3;                       // this lane's bins lo..lo+3; lane 0 holds the highest
    const uint4 v = *reinterpret_cast<const uint4*>(hist + lo);
    const unsigned ls = v.x + v.y + v.z + v.w;
    const unsigned blk = __reduce_add_sync(0xffffffffu, ls);
    if (cum + blk >= (unsigned)need) {
      unsigned incl = ls;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
      }
      const int L = __ffs(__ballot_sync(0xffffffffu, cum + incl >= (unsigned)need)) - 1;
      unsigned c = cum + incl - ls;                           // elements above this lane's bins
      int b = lo, above = 0, cnt = 0;
      const unsigned bv[4] = {v.w, v.z, v.y, v.x};            // bins lo+3 .. lo
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (cnt == 0 && c + bv[i] >= (unsigned)need) { b = lo + 3 - i; above = (int)c; cnt = (int)bv[i]; }
        else if (cnt == 0) c += bv[i];
      bin_out = __shfl_sync(0xffffffffu, b, L);
      above_out = __shfl_sync(0xffffffffu, above, L);
      count_out = __shfl_sync(0xffffffffu, cnt, L);
      return;
    }
    cum += blk;
  }
}

// Cluster-wide pivot search over the CTAs' NB-bin histograms (complete and visible cluster-wide on entry): the bin
// holding the need-th largest element counted from the top bin, and the number of elements in the bins above it.
// Every CTA returns the same result. CS == 1 reads its own histogram and uses block barriers only; CS > 1 sums this
// CTA's slice of the bins over the cluster into s_slice first.
__device__ void pivot_round(cg::cluster_group& cluster, int CS, int crank, const unsigned* s_hist, unsigned* s_slice,
                            int* s_sltot, int* s_piv, int* s_ws, int NB, int need, int& bin_out, int& above_out) {
  const int tid = threadIdx.x;
  const int SL = NB / CS, s0 = crank * SL;
  const unsigned* sl = s_hist;
  if (CS > 1) {
    for (int i = tid; i < SL; i += kThreads) {
      unsigned v = 0;
      for (int c = 0; c < CS; ++c) v += cluster.map_shared_rank(s_hist, c)[s0 + i];
      s_slice[i] = v;
    }
    __syncthreads();
    sl = s_slice;
  }
  const int BPT = (SL + kThreads - 1) / kThreads;
  int lsum = 0;
  for (int i = 0; i < BPT; ++i) {
    const int bin = tid * BPT + i;
    if (bin < SL) lsum += (int)sl[bin];
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
        const int hv = (int)sl[bin];
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
__global__ void __launch_bounds__(kThreads, 2) sparse_step_kernel(const DecodeParams p,
                                                                   const __grid_constant__ CUtensorMap zmap) {
  unsigned char* dsm = g_dsm;
  __shared__ __align__(8) uint64_t s_full[kMaxRing];
  __shared__ uint32_t s_taddr;
  __shared__ __align__(16) float s_u[kMaxR];
  __shared__ float s_pre[kWarps * 32];
  __shared__ int s_sltot[kMaxCluster];
  __shared__ int s_cgt[kMaxCluster], s_ceq[kMaxCluster], s_cflag[kMaxCluster];
  __shared__ int s_piv[4];
  __shared__ int s_ws[kWarps];
  __shared__ int s_fpre;
  __shared__ long long s_segoff;
  __shared__ float s_m[HP], s_l[HP];
  __shared__ float s_acc[HP * kHeadDim];

  cg::cluster_group cluster = cg::this_cluster();
  const int CS = (int)cluster.num_blocks();
  const int crank = (int)cluster.block_rank();
  const int seg = blockIdx.y;
  const int b = seg / p.G, g = seg - b * p.G;
  const int tid = threadIdx.x;
  // dynamic shared memory: [histogram | cluster slice | selection bitmaps | candidate list] aliasing [attend engine],
  // then the attend row list
  unsigned* s_hist = reinterpret_cast<unsigned*>(dsm);
  unsigned* s_slice = reinterpret_cast<unsigned*>(dsm + 4096 * 4);
  uint32_t* s_gt = reinterpret_cast<uint32_t*>(dsm + p.bm_off);
  uint32_t* s_eq = s_gt + p.nwp;
  const uint32_t* s_lkey = reinterpret_cast<const uint32_t*>(dsm + p.list_off);
  const uint32_t* s_lcol = s_lkey + p.cap;
  uint32_t* s_arow = reinterpret_cast<uint32_t*>(dsm + p.union_bytes);
  uint32_t* s_skey = p.keys_out ? reinterpret_cast<uint32_t*>(dsm + p.skey_off) : nullptr;   // [column - kb]
#define CSYNC() do { if (CS > 1) cluster.sync(); else __syncthreads(); } while (0)

  const int c0 = p.lo + crank * p.cpc;
  const int c1 = min(p.hi, c0 + p.cpc);
  const int nloc = max(0, c1 - c0);
  const int kb = (c0 / 32) * 32;                        // bitmap bit i and list column i stand for column kb + i

  // ---------------- prologue: z column (rank 0 of the cluster) and u ----------------
  // resident-key scan: the ring's barriers and 256 TMEM columns, then the first tiles go in flight before u is known
  const bool tkl = p.tkeys && p.select_mode == 1 && p.scan;   // launch-uniform: decides cluster-wide control flow
  const bool tk = tkl && nloc > 0;                              // this CTA holds keys in TMEM
  if (tk) {
    if (tid == 0) {
      for (int i = 0; i < p.nring; ++i) mbar_init(&s_full[i], 1);
      mbar_init_fence();
    }
    if (tid < 32) { tmem_alloc(&s_taddr, kTmemCols); tmem_relinquish(); }
  }
  if (p.select_mode == 1) {
    for (int i = tid; i < (tk ? 2048 : 4096); i += kThreads) s_hist[i] = 0u;   // tk: the packed scan histogram
    if (!tk) for (int i = tid; i < 2 * p.nwp; i += kThreads) s_gt[i] = 0u;   // s_eq follows s_gt (tk: after the scan)
    if (tid == 0) { g_list_count = 0u; g_list_thr = 0u; }
  }
  if (tk) {
    tmem_fence_before_sync();
    __syncthreads();
    tmem_fence_after_sync();
  }
  const TKeyGeo<IDX_T> tg(c0, c1, tk ? s_taddr : 0u);
  if (tk && tid == 0)
    for (int t = 0; t < p.nring && t < tg.ntiles; ++t) tkey_issue(tg, &zmap, dsm + p.ring_off, s_full, p.nring, seg * p.r, t);
  if (p.k_new && crank == 0) write_z_column<IDX_T>(p, b, g);
  // selection-independent inputs of the compaction, loaded while the scan's first loads are in flight (at once when
  // this CTA scans nothing): the segment's first candidate row, this CTA's share of F into the attend list, and
  // (canonical order) how many F rows precede the candidates. With F <= kThreads (one row per thread) the loads are
  // issued before u is computed and consumed after it, so the two latencies overlap.
  const auto load_rows = [&](auto&& between) {
    const int F = p.F;
    const int fsh0 = (crank * F) / CS, fshare = ((crank + 1) * F) / CS - fsh0;
    if (F <= kThreads) {
      const long long fr = tid < F ? p.fixed_rows[(size_t)seg * F + tid] : 0;
      const long long so0 = p.off_lo[seg];
      between();
      if (tid >= fsh0 && tid < fsh0 + fshare) s_arow[tid - fsh0] = checked_row(fr, p.total_rows, p.err);
      const int fp = __syncthreads_count(p.canonical && tid < F && fr < so0);
      if (tid == 0) { s_segoff = so0; s_fpre = fp; }
    } else {
      between();
      for (int i = tid; i < fshare; i += kThreads)
        s_arow[i] = checked_row(p.fixed_rows[(size_t)seg * F + fsh0 + i], p.total_rows, p.err);
      if (tid < 32) {
        const long long so0 = p.off_lo[seg];
        int fp = 0;
        if (p.canonical)
          for (int base = 0; base < F; base += 32) {
            const int i = base + tid;
            fp += __popc(__ballot_sync(0xffffffffu, i < F && p.fixed_rows[(size_t)seg * F + i] < so0));
          }
        if (tid == 0) { s_segoff = so0; s_fpre = fp; }
      }
    }
  };
  // u is computed inside the scan, under its first loads (compute_u ends with the __syncthreads() that also
  // publishes the cleared histogram before any key is counted); a CTA without columns needs no u
  const auto pre_u = [&]() { load_rows([&]() { compute_u<IDX_T>(p, b, g, s_u, s_pre); }); };
  const bool scans = p.scan && nloc > 0 && !tk;
  if (!scans && !tk) load_rows([]() {});

  // ---------------- scan: candidate scores -> order keys ----------------
  float* so = p.scores_out ? p.scores_out + (size_t)seg * p.M - p.lo : nullptr;   // indexed by column
  const ZSrc zsrc{reinterpret_cast<const IDX_T*>(p.zT) + (size_t)seg * p.r * p.C, p.r, p.C, p.zvec};
  if (tk) {
    pre_u();                                               // ends with __syncthreads(): u and the cleared histogram
    if (!tkey_scan<IDX_T>(tg, &zmap, dsm + p.ring_off, s_full, p.nring, seg * p.r, s_u, s_hist, so))
      atomicOr(p.err, kErrWaitLimit);
    tmem_wait_st();
    tmem_fence_before_sync();
    __syncthreads();
    tmem_fence_after_sync();
    // unpack the 16-bit bin pairs into the 4096-word histogram (over the packed words and the ring's first stage,
    // both free now), and clear the bitmaps, which reuse the ring too
    uint32_t hp[2048 / kThreads];
#pragma unroll
    for (int i = 0; i < 2048 / kThreads; ++i) hp[i] = s_hist[tid + i * kThreads];
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 2048 / kThreads; ++i) {
      const int wi = tid + i * kThreads;
      s_hist[2 * wi] = hp[i] & 0xffffu;
      s_hist[2 * wi + 1] = hp[i] >> 16;
    }
    for (int i = tid; i < 2 * p.nwp; i += kThreads) s_gt[i] = 0u;
  } else if (scans) {
    if (p.select_mode == 1) {
      if (so) {
        SinkFirst<true> sk{so, p.list_off, p.cap, p.k, kb};
        scan_columns<IDX_T>(zsrc, c0, c1, s_u, sk, pre_u);
      } else {
        SinkFirst<false> sk{nullptr, p.list_off, p.cap, p.k, kb};
        scan_columns<IDX_T>(zsrc, c0, c1, s_u, sk, pre_u);
      }
    } else if (s_skey) {
      SinkKeys sk{s_skey, kb, so};
      scan_columns<IDX_T>(zsrc, c0, c1, s_u, sk, pre_u);
    } else {
      SinkScores sk{so};
      scan_columns<IDX_T>(zsrc, c0, c1, s_u, sk, pre_u);
    }
  }
  CSYNC();

  // ---------------- radix select of the k-th largest key over the cluster ----------------
  // 1) the histogram of the top 12 key bits gives the pivot bin b0; the candidate list holds every key of bin >= b0
  //    (the scan's threshold never passed b0);
  // 2) two 10-bit passes over the list's keys of bin b0 find the exact k-th key tau and how many of its copies
  //    (k_rem, in position order) complete the top-k;
  // 3) the chosen columns are marked in two bitmaps (key > tau, key == tau).
  // If some CTA's list overflowed (heavy ties), steps 2-3 rescan the index columns instead of reading the list.
  uint32_t tau = 0;
  int k_rem = 0;
  bool selected = false;
  if (p.select_mode == 1 && CS == 1 && (tkl || g_list_count <= (unsigned)p.cap)) {
    // One CTA, list complete: one warp finds the pivot bin from the histogram; if that bin holds at most kSmall
    // keys, one list pass marks every key above it and gathers the bin's keys, and two radix passes over the
    // gathered keys alone find the exact k-th key.
    constexpr int kSmall = 1024;
    if (tid < 32) {
      int b0, gt0, n0;
      warp_pivot4096(s_hist, p.k, b0, gt0, n0);
      if (tid == 0) { s_piv[0] = b0; s_piv[1] = gt0; s_piv[2] = n0; }
    }
    __syncthreads();
    const int b0 = s_piv[0], gt0 = s_piv[1], n0 = s_piv[2];
    // resident keys: compact every key of bin >= b0 (about k + n0 of them) into the candidate list -- a count
    // sweep, a block scan for each warp's first slot, a write sweep whose slots come from warp votes (warp-uniform
    // branches only) -- so the list path below runs on it; if the list region cannot hold them, the general path
    // re-reads the keys from TMEM instead
    bool have = n0 <= kSmall;
    int n_list = tkl ? 0 : (int)g_list_count;
    if (tk && have) {
      int nge = 0;
      tg.for_each_chunk([&](const uint32_t (&r)[8], int) {
#pragma unroll
        for (int e = 0; e < 8; ++e) nge += (int)((int)(r[e] >> 20) >= b0);
      });
      int tot;
      const int incl = block_inclusive_scan(nge, s_ws, &tot);
      have = tot <= p.cap;                               // CTA-uniform
      if (have) {
        uint32_t* lk = reinterpret_cast<uint32_t*>(dsm + p.list_off);
        uint32_t* lc = lk + p.cap;
        const int lane = tid & 31;
        int base = __shfl_sync(0xffffffffu, incl - nge, 0);   // the warp's first slot (threads are warp-major)
        tg.for_each_chunk([&](const uint32_t (&r)[8], int i0) {
          // one warp scan per chunk of 8 keys: this lane's matches go to consecutive slots after the lower lanes'
          unsigned m = 0u;
#pragma unroll
          for (int e = 0; e < 8; ++e) m |= ((int)(r[e] >> 20) >= b0 ? 1u : 0u) << e;
          const int c = __popc(m);
          int x = c;
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
          }
          int o = base + x - c;
          base += __shfl_sync(0xffffffffu, x, 31);
          if (m) {
            const int cb = tg.col(i0) - kb;               // key i0 + e sits at column cb + colstep(e)
#pragma unroll
            for (int e = 0; e < 8; ++e)
              if ((m >> e) & 1u) { lk[o] = r[e]; lc[o] = (uint32_t)(cb + tg.colstep(e)); ++o; }
          }
        });
        n_list = tot;
      }
    }
    if (have) {
      uint32_t* skey = s_hist;                           // [kSmall] keys of bin b0, then [kSmall] their columns
      uint32_t* scol = s_hist + kSmall;
      unsigned* whist = s_hist + 2 * kSmall;             // [1024] digit histogram of the gathered keys
      if (tid == 0) g_list_thr = 0u;                     // reused as the gathered keys' fill counter
      __syncthreads();
      const unsigned lt = (1u << (tid & 31)) - 1u;
      constexpr int U = 4;                               // list entries per thread and step, loads batched
      for (int base = 0; base < n_list; base += U * kThreads) {   // uniform trip count: warp-aggregated appends
        uint32_t key[U];
#pragma unroll
        for (int j = 0; j < U; ++j) {
          const int i = base + j * kThreads + tid;
          key[j] = i < n_list ? s_lkey[i] : 0u;
        }
        unsigned bal[U], tot = 0;
#pragma unroll
        for (int j = 0; j < U; ++j) {
          const int i = base + j * kThreads + tid;
          const int bin = (int)(key[j] >> 20);
          if (i < n_list && bin > b0) {
            const uint32_t c = s_lcol[i];
            atomicOr(&s_gt[c >> 5], 1u << (c & 31));
            if (s_skey) s_skey[c] = key[j];
          }
          bal[j] = __ballot_sync(0xffffffffu, i < n_list && bin == b0);
          tot += __popc(bal[j]);
        }
        if (tot) {                                       // one shared atomic per warp and step
          unsigned o = 0;
          if ((tid & 31) == 0) o = atomicAdd(&g_list_thr, tot);
          o = __shfl_sync(0xffffffffu, o, 0);
#pragma unroll
          for (int j = 0; j < U; ++j) {
            if ((bal[j] >> (tid & 31)) & 1u) {
              const unsigned slot = o + __popc(bal[j] & lt);
              skey[slot] = key[j];
              scol[slot] = s_lcol[base + j * kThreads + tid];
            }
            o += __popc(bal[j]);
          }
        }
      }
      __syncthreads();
      // two 10-bit refinement passes over the gathered keys only (block histogram + block pivot search)
      uint32_t prefix = (uint32_t)b0 << 20, pmask = 0xfff00000u;
      int need = p.k - gt0;
#pragma unroll 1
      for (int pass = 0; pass < 2; ++pass) {
        const int shift = pass == 0 ? 10 : 0;
        for (int i = tid; i < 1024; i += kThreads) whist[i] = 0u;
        __syncthreads();
        for (int i = tid; i < n0; i += kThreads) {
          const uint32_t key = skey[i];
          if ((key & pmask) == prefix) atomicAdd(&whist[(key >> shift) & 1023u], 1u);
        }
        __syncthreads();
        int bn, above;
        pivot_round(cluster, 1, 0, whist, nullptr, s_sltot, s_piv, s_ws, 1024, need, bn, above);
        prefix |= (uint32_t)bn << shift;
        pmask |= 1023u << shift;
        need -= above;
      }
      for (int i = tid; i < n0; i += kThreads) {
        const uint32_t key = skey[i], c = scol[i];
        if (key > prefix) atomicOr(&s_gt[c >> 5], 1u << (c & 31));
        else if (key == prefix) atomicOr(&s_eq[c >> 5], 1u << (c & 31));
        if (s_skey && key >= prefix) s_skey[c] = key;
      }
      __syncthreads();
      tau = prefix;
      k_rem = need;
      selected = true;
    }
  }
  if (p.select_mode == 1 && !selected) {
    int b0, gt0;
    pivot_round(cluster, CS, crank, s_hist, s_slice, s_sltot, s_piv, s_ws, 4096, p.k, b0, gt0);
    const unsigned cnt = g_list_count;
    bool use_list;
    if (tkl) {
      use_list = false;                                  // every CTA's keys are in its TMEM
    } else if (CS > 1) {
      if (tid < CS) cluster.map_shared_rank(s_cflag, tid)[crank] = cnt > (unsigned)p.cap ? 1 : 0;
      cluster.sync();
      use_list = true;
      for (int c = 0; c < CS; ++c) use_list = use_list && s_cflag[c] == 0;
    } else {
      use_list = cnt <= (unsigned)p.cap;
    }
    const int n_list = use_list ? (int)cnt : 0;
    uint32_t prefix = (uint32_t)b0 << 20, pmask = 0xfff00000u;
    k_rem = p.k - gt0;
    // passes 0 and 1: digits 19..10 and 9..0 of the keys under the prefix; pass 2: the marks
#pragma unroll 1
    for (int pass = 0; pass < 3; ++pass) {
      const int shift = pass == 0 ? 10 : 0;
      if (pass < 2) {
        for (int i = tid; i < 1024; i += kThreads) s_hist[i] = 0u;
        __syncthreads();
      }
      if (tkl) {
        if (tk)
          tg.for_each_chunk([&](const uint32_t (&r)[8], int i0) {
#pragma unroll
            for (int e = 0; e < 8; ++e) {                // prefix >= 7 << 20: key 0 (no candidate) never matches
              const uint32_t key = r[e];
              if (pass < 2) {
                if ((key & pmask) == prefix) atomicAdd(&s_hist[(key >> shift) & 1023u], 1u);
              } else if (key >= prefix) {
                const uint32_t c = (uint32_t)(tg.col(i0 + e) - kb);
                atomicOr(key > prefix ? &s_gt[c >> 5] : &s_eq[c >> 5], 1u << (c & 31));
                if (s_skey) s_skey[c] = key;
              }
            }
          });
      } else if (use_list) {
        for (int i = tid; i < n_list; i += kThreads) {
          const uint32_t key = s_lkey[i];
          if (pass < 2) {
            if ((key & pmask) == prefix) atomicAdd(&s_hist[(key >> shift) & 1023u], 1u);
          } else if (key >= prefix) {
            const uint32_t c = s_lcol[i];
            atomicOr(key > prefix ? &s_gt[c >> 5] : &s_eq[c >> 5], 1u << (c & 31));
            if (s_skey) s_skey[c] = key;
          }
        }
      } else if (nloc > 0) {
        SinkRescan sk{pass == 2, s_hist, prefix, pmask, shift, s_gt, s_eq, prefix, kb, s_skey};
        scan_columns<IDX_T>(zsrc, c0, c1, s_u, sk);
      }
      if (pass < 2) {
        CSYNC();
        int bn, above;
        pivot_round(cluster, CS, crank, s_hist, s_slice, s_sltot, s_piv, s_ws, 1024, k_rem, bn, above);
        prefix |= (uint32_t)bn << shift;
        pmask |= 1023u << shift;
        k_rem -= above;
      }
    }
    tau = prefix;
    __syncthreads();
  }

  if (tk) {                                              // every key has been read back: release the TMEM
    tmem_fence_before_sync();
    __syncthreads();
    if (tid < 32) tmem_dealloc(s_taddr, kTmemCols);
  }

  // ---------------- ordered selection: chosen candidates in ascending position order ----------------
  const long long seg_off = s_segoff;
  const int F = p.F;
  const int fsh0 = (crank * F) / CS, fshare = ((crank + 1) * F) / CS - fsh0;
  const int out_base = p.canonical ? s_fpre : F;
  long long* ro = p.rows_out ? p.rows_out + (size_t)seg * p.S + out_base : nullptr;
  int n_sel = 0;
  if (p.select_mode == 2) {
    // every candidate: column c has rank c - lo
    n_sel = nloc;
    for (int c = c0 + tid; c < c1; c += kThreads) {
      const long long row = seg_off + (long long)(c - p.lo);
      if (ro) ro[c - p.lo] = row;
      if (p.keys_out) p.keys_out[(size_t)seg * p.kst + (c - p.lo)] = pack_key64(s_skey[c - kb], p.key_pos + c);
      s_arow[fshare + (c - c0)] = checked_row(row, p.total_rows, p.err);
    }
  } else if (p.select_mode == 1) {
    // this thread's run of bitmap words (odd run length: the 8 threads of a quarter warp hit different banks)
    const int nw = nloc > 0 ? (c1 - kb + 31) >> 5 : 0;
    const int EPT = ((nw + kThreads - 1) / kThreads) | 1;
    const int tw0 = min(nw, tid * EPT), tw1 = min(nw, tw0 + EPT);
    int cgt = 0, ceq = 0;
    for (int w = tw0; w < tw1; ++w) {
      cgt += __popc(s_gt[w]);
      ceq += __popc(s_eq[w]);
    }
    // packed block scan of (gt, eq) counts: both stay below 2^16 per CTA
    const unsigned packed = (unsigned)cgt | ((unsigned)ceq << 16);
    int tot;
    const unsigned inc = (unsigned)block_inclusive_scan((int)packed, s_ws, &tot);
    const int ex_gt = (int)((inc - packed) & 0xffffu), ex_eq = (int)((inc - packed) >> 16);
    const int tot_gt = (int)((unsigned)tot & 0xffffu), tot_eq = (int)((unsigned)tot >> 16);
    int eo = 0, so_r = 0;                       // ties and selections before this CTA
    if (CS > 1) {
      if (tid < CS) {
        cluster.map_shared_rank(s_cgt, tid)[crank] = tot_gt;
        cluster.map_shared_rank(s_ceq, tid)[crank] = tot_eq;
      }
      cluster.sync();
      for (int c = 0; c < crank; ++c) { so_r += s_cgt[c]; eo += s_ceq[c]; }
      so_r += min(max(k_rem, 0), eo);
    }
    const int sel_off = so_r;                   // this CTA's first rank
    n_sel = tot_gt + min(max(k_rem - eo, 0), tot_eq);
    int er = eo + ex_eq;                        // tie rank of this thread's first equal key
    int rank = so_r + ex_gt + min(max(k_rem - eo, 0), ex_eq);
    for (int w = tw0; w < tw1; ++w) {
      const uint32_t gw = s_gt[w];
      uint32_t m = gw | s_eq[w];
      while (m) {
        const int bit = __ffs(m) - 1;
        m &= m - 1u;
        bool take = true;
        if (!((gw >> bit) & 1u)) take = er++ < k_rem;
        if (take) {
          const long long row = seg_off + (long long)(kb + 32 * w + bit - p.lo);
          if (ro) ro[rank] = row;
          if (p.keys_out)
            p.keys_out[(size_t)seg * p.kst + rank] = pack_key64(s_skey[32 * w + bit], p.key_pos + kb + 32 * w + bit);
          s_arow[fshare + (rank - sel_off)] = checked_row(row, p.total_rows, p.err);
          ++rank;
        }
      }
    }
  }
  if (p.keys_out && crank == 0)
    for (int i = p.k + tid; i < p.kst; i += kThreads) p.keys_out[(size_t)seg * p.kst + i] = 0ull;   // below every key
  __syncthreads();
  if (p.rows_out && crank == 0 && tid < 32) {
    // F into the row list: first (reference order), or around the candidates when canonical
    const int lane = tid;
    long long* rf = p.rows_out + (size_t)seg * p.S;
    const long long* fr = p.fixed_rows + (size_t)seg * F;
    if (!p.canonical) {
      for (int i = lane; i < F; i += 32) rf[i] = fr[i];
    } else {
      int nlo = 0, nhi = 0;
      const unsigned lt = (1u << lane) - 1u;
      for (int base = 0; base < F; base += 32) {
        const int i = base + lane;
        const long long v = i < F ? fr[i] : 0;
        const bool lo_side = i < F && v < seg_off, hi_side = i < F && v >= seg_off;
        const unsigned ml = __ballot_sync(0xffffffffu, lo_side), mh = __ballot_sync(0xffffffffu, hi_side);
        if (lo_side) rf[nlo + __popc(ml & lt)] = v;
        if (hi_side) rf[s_fpre + p.k + nhi + __popc(mh & lt)] = v;
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
  int skip_neg;           // mode 0: a negative row id marks a row that is not read (no error)
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
__global__ void __launch_bounds__(kThreads, 2) attend_kernel(const AttendParams p) {
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
    for (int i = threadIdx.x; i < r1 - r0; i += kThreads) {
      const long long row = p.rows[(size_t)seg * p.S + r0 + i];
      s_arow[i] = (p.skip_neg && row < 0) ? 0xffffffffu : checked_row(row, p.total_rows, p.err);
    }
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
