// Indexer and cache-append kernels: the standalone forms of project_keys / project_queries / candidate_scores
// (attention-lab indexer.py:15-29) and of LabCache.append (qwen_wrap.py:90-106), with the prefill index-table build
// (z = Wk . k_pre for every new position, qwen_wrap.py:320-324) fused into the same launch as the K/V copy.
#pragma once
#include "al_common.cuh"

namespace al {

// ------------------------------------------------------------------------------------------------ append
// k_cache/v_cache [B,G,C,d] <- k_new/v_new [B,G,T,d] (element strides) at positions [start, start+T).
// z (optional): zT [B,G,r,C] columns [start, start+T) <- either given z values [B,G,r,T] (strided) or, when wk is
// given, Wk[g] . k_pre[b,g,t] computed here from k_pre [B,G,T,d] (strided).
struct AppendParams {
  int B, G, C, T, r, start;
  void* k_cache; void* v_cache;
  const void* k_new; long long kn_s[4];
  const void* v_new; long long vn_s[4];
  void* zT;
  const void* z_new; long long zn_s[4];
  const void* k_pre; long long kp_s[4];
  const void* wk;
};

template <typename DST, typename SRC>
__global__ void __launch_bounds__(kThreads) append_kv_kernel(const AppendParams p) {
  const long long total = (long long)p.B * p.G * p.T * kHeadDim;
  for (long long i = blockIdx.x * (long long)kThreads + threadIdx.x; i < total; i += (long long)gridDim.x * kThreads) {
    const int e = (int)(i % kHeadDim);
    long long rest = i / kHeadDim;
    const int t = (int)(rest % p.T); rest /= p.T;
    const int g = (int)(rest % p.G);
    const int b = (int)(rest / p.G);
    const size_t dst = (((size_t)b * p.G + g) * p.C + p.start + t) * kHeadDim + e;
    const SRC* kn = reinterpret_cast<const SRC*>(p.k_new);
    const SRC* vn = reinterpret_cast<const SRC*>(p.v_new);
    reinterpret_cast<DST*>(p.k_cache)[dst] =
        fromf<DST>(tof(kn[b * p.kn_s[0] + g * p.kn_s[1] + t * p.kn_s[2] + e * p.kn_s[3]]));
    reinterpret_cast<DST*>(p.v_cache)[dst] =
        fromf<DST>(tof(vn[b * p.vn_s[0] + g * p.vn_s[1] + t * p.vn_s[2] + e * p.vn_s[3]]));
  }
}

// Given z values: zT[b,g,j,start+t] = z_new[b,g,j,t].
template <typename ZT, typename ZS>
__global__ void __launch_bounds__(kThreads) append_z_copy_kernel(const AppendParams p) {
  const long long total = (long long)p.B * p.G * p.r * p.T;
  for (long long i = blockIdx.x * (long long)kThreads + threadIdx.x; i < total; i += (long long)gridDim.x * kThreads) {
    const int t = (int)(i % p.T);
    long long rest = i / p.T;
    const int j = (int)(rest % p.r); rest /= p.r;
    const int g = (int)(rest % p.G);
    const int b = (int)(rest / p.G);
    const ZS* zn = reinterpret_cast<const ZS*>(p.z_new);
    reinterpret_cast<ZT*>(p.zT)[(((size_t)b * p.G + g) * p.r + j) * p.C + p.start + t] =
        fromf<ZT>(tof(zn[b * p.zn_s[0] + g * p.zn_s[1] + j * p.zn_s[2] + t * p.zn_s[3]]));
  }
}

// Index-table build from k_pre: one CTA per (b, g, 32 positions). wk[g] and the 32 k_pre rows are staged in shared
// memory as fp32; thread (tx, ty) computes z for position tx and index rows ty, ty+8, ty+16, ty+24.
// Writes are coalesced along the position axis of zT [B,G,r,C].
template <typename IDX_T>
__global__ void __launch_bounds__(kThreads) project_keys_kernel(const AppendParams p) {
  __shared__ float s_w[kMaxR][kHeadDim + 1];
  __shared__ float s_k[32][kHeadDim + 1];
  const int seg = blockIdx.y, b = seg / p.G, g = seg - b * p.G;
  const int t0 = blockIdx.x * 32;
  const IDX_T* wk = reinterpret_cast<const IDX_T*>(p.wk) + (size_t)g * p.r * kHeadDim;
  const IDX_T* kp = reinterpret_cast<const IDX_T*>(p.k_pre) + b * p.kp_s[0] + g * p.kp_s[1];
  for (int i = threadIdx.x; i < kMaxR * kHeadDim; i += kThreads) {
    const int j = i / kHeadDim, e = i % kHeadDim;
    s_w[j][e] = j < p.r ? tof(wk[(size_t)j * kHeadDim + e]) : 0.f;
  }
  for (int i = threadIdx.x; i < 32 * kHeadDim; i += kThreads) {
    const int t = i / kHeadDim, e = i % kHeadDim;
    s_k[t][e] = (t0 + t < p.T) ? tof(kp[(t0 + t) * p.kp_s[2] + e * p.kp_s[3]]) : 0.f;
  }
  __syncthreads();
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  if (t0 + tx >= p.T) return;
  IDX_T* zT = reinterpret_cast<IDX_T*>(p.zT) + (size_t)seg * p.r * p.C + p.start + t0 + tx;
  for (int j = ty; j < p.r; j += kWarps) {
    float a = 0.f;
#pragma unroll 16
    for (int e = 0; e < kHeadDim; ++e) a = fmaf(s_w[j][e], s_k[tx][e], a);
    zT[(size_t)j * p.C] = fromf<IDX_T>(a);
  }
}

// ------------------------------------------------------------------------------------------------ u and scores
struct IndexParams {
  int B, G, h, T, r, C, lo, hi;
  const void* q_pre; long long qp_s[5];   // [B,G,h,T,d]
  const void* wq_t;                       // [G,h*d,r]
  const void* u; long long u_s[4];        // [B,G,T,r]
  const void* zT;                         // [B,G,r,C]
  void* out;                              // u [B,G,T,r] or scores [B,G,T,M] (contiguous)
  int out_f32;                            // write fp32 instead of the index dtype
};

// u[b,g,t,:] = concat_h(q_pre[b,g,:,t,:]) . wq_t[g]: one CTA per (b,g,t).
template <typename IDX_T>
__global__ void __launch_bounds__(kThreads) project_queries_kernel(const IndexParams p) {
  __shared__ float s_pre[kWarps * 32];
  const int bgt = blockIdx.x;
  const int t = bgt % p.T, g = (bgt / p.T) % p.G, b = bgt / (p.T * p.G);
  const IDX_T* qp = reinterpret_cast<const IDX_T*>(p.q_pre) + b * p.qp_s[0] + g * p.qp_s[1] + t * p.qp_s[3];
  const int hd = p.h * kHeadDim;
  const IDX_T* wq = reinterpret_cast<const IDX_T*>(p.wq_t) + (size_t)g * hd * p.r;
  const int j = threadIdx.x & 31, w = threadIdx.x >> 5;
  float acc = 0.f;
  if (j < p.r) {
#pragma unroll 8
    for (int f = w; f < hd; f += kWarps)
      acc = fmaf(tof(qp[(f / kHeadDim) * p.qp_s[2] + (f % kHeadDim) * p.qp_s[4]]), tof(wq[(size_t)f * p.r + j]), acc);
  }
  s_pre[w * 32 + j] = acc;
  __syncthreads();
  if (threadIdx.x < p.r) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kWarps; ++i) s += s_pre[i * 32 + threadIdx.x];
    const size_t o = (size_t)bgt * p.r + threadIdx.x;
    if (p.out_f32) reinterpret_cast<float*>(p.out)[o] = s;
    else reinterpret_cast<IDX_T*>(p.out)[o] = fromf<IDX_T>(s);
  }
}

// scores[b,g,t,m] = u[b,g,t,:] . zT[b,g,:,lo+m]: grid (column blocks, B*G*T); one column per thread, coalesced
// along the column axis, r rows of zT per column.
template <typename IDX_T>
__global__ void __launch_bounds__(kThreads) candidate_scores_kernel(const IndexParams p) {
  __shared__ float s_u[kMaxR];
  const int bgt = blockIdx.y;
  const int t = bgt % p.T, g = (bgt / p.T) % p.G, b = bgt / (p.T * p.G);
  const IDX_T* u = reinterpret_cast<const IDX_T*>(p.u) + b * p.u_s[0] + g * p.u_s[1] + t * p.u_s[2];
  if (threadIdx.x < kMaxR) s_u[threadIdx.x] = threadIdx.x < p.r ? tof(u[threadIdx.x * p.u_s[3]]) : 0.f;
  __syncthreads();
  const int M = p.hi - p.lo;
  const int m = blockIdx.x * kThreads + threadIdx.x;
  if (m >= M) return;
  const IDX_T* z = reinterpret_cast<const IDX_T*>(p.zT) + ((size_t)b * p.G + g) * p.r * p.C + p.lo + m;
  float a = 0.f;
  for (int j = 0; j < p.r; ++j) a = fmaf(s_u[j], tof(z[(size_t)j * p.C]), a);
  const size_t o = (size_t)bgt * M + m;
  if (p.out_f32) reinterpret_cast<float*>(p.out)[o] = a;
  else reinterpret_cast<IDX_T*>(p.out)[o] = fromf<IDX_T>(a);
}

}  // namespace al
