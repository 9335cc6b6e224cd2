// tn_attn.cu -- one-query GQA decode attention over the KV cache.
//
// The attention of web/inference-worker.js:556-564 (scores q.k / sqrt(hd),
// softmax over the row's cached positions, weighted sum of V) for T query
// rows at once, each row over its own sequence slot and length.  The cache
// holds f32 rows (the reference's format, :554 and :640-653) or, opt-in,
// fp16 or fp8 e4m3 rows (half / a quarter of the bytes; values rounded to
// nearest even on append, e4m3 saturating at +-448).
//
// Work split.  CTA (split, KV head, row) streams its share of the row's
// positions; the split count S is chosen so that the grid fills every SM
// (one decoding row of an 8-KV-head model is 8 x S CTAs), and a row shorter
// than S splits of two warp steps per warp uses fewer (the grid is fixed for
// a captured step; the row lengths are not).  Within a CTA each
// of the 8 warps takes a contiguous part of that share.  A lane holds HD/32
// dimensions of q for the G query heads of the KV head; a warp step covers
// PS = 32/G positions: the PS x G partial dot products of a lane are
// reduce-scattered over the warp so that lane l ends with the full score of
// (position l / G, head l % G) -- every exp is computed once -- and an online
// softmax per head rescales the lane's G x HD/32 output accumulators.  The
// warps merge in shared memory.  With one split the CTA writes the output;
// otherwise it writes its partial (unnormalised output, running max and sum
// per head) to a workspace, and the CTA that arrives last at the (row, KV
// head) -- a release / acquire counter -- merges the S partials in split
// order (deterministic) and resets the counter for the next launch.  Up to
// 8 splits, and any split count over caches of at most 4096 positions, run as
// one thread-block cluster per (row, KV head) and merge through distributed
// shared memory instead (no global round trip: the decode chain's short rows
// are latency-bound), also in split order.
#include <atomic>
#include <cfloat>

#include <cooperative_groups.h>
#include <cuda_fp16.h>

#include "tn_kernels.cuh"
#include "tn_ptx.cuh"

namespace cg = cooperative_groups;

namespace tn {

constexpr int ATT_WARPS = 8;
constexpr int ATT_THREADS = ATT_WARPS * 32;
constexpr int ATT_MAX_SPLITS = 32;
constexpr int kAttnClusterCtx = 4096;  // caches up to this long merge splits within a cluster

struct AttnArgs {
  const float* q;
  int ldq;
  const void* kc;  // KT elements
  const void* vc;
  KvMap kv;  // the rows' places in the cache
  const RowInfo* rows;
  int S, nkv;
  float scale;
  float* out;
  int ldo;
  float* ws;  // partials [row][KV head][split][pstride] (S > 1)
  int* cnt;   // arrivals per (row, KV head), zero between launches (S > 1)
  int pstride;
};

// floats of one partial: G x HD outputs, G maxima, G sums (16-byte multiple)
__host__ __device__ constexpr int attn_pstride(int G, int HD) { return (G * HD + 2 * G + 3) / 4 * 4; }

// DPL consecutive elements of a cached row, as floats
template <typename KT, int DPL>
struct KvVec;
template <>
struct KvVec<float, 4> {
  using Raw = float4;
  static __device__ __forceinline__ Raw load(const float* p) { return *reinterpret_cast<const float4*>(p); }
  static __device__ __forceinline__ void cvt(const Raw& r, float (&o)[4]) {
    o[0] = r.x;
    o[1] = r.y;
    o[2] = r.z;
    o[3] = r.w;
  }
};
template <>
struct KvVec<float, 2> {
  using Raw = float2;
  static __device__ __forceinline__ Raw load(const float* p) { return *reinterpret_cast<const float2*>(p); }
  static __device__ __forceinline__ void cvt(const Raw& r, float (&o)[2]) {
    o[0] = r.x;
    o[1] = r.y;
  }
};
template <>
struct KvVec<float, 1> {
  using Raw = float;
  static __device__ __forceinline__ Raw load(const float* p) { return *p; }
  static __device__ __forceinline__ void cvt(const Raw& r, float (&o)[1]) { o[0] = r; }
};
template <>
struct KvVec<__half, 4> {
  using Raw = uint2;
  static __device__ __forceinline__ Raw load(const __half* p) { return *reinterpret_cast<const uint2*>(p); }
  static __device__ __forceinline__ void cvt(const Raw& r, float (&o)[4]) {
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&r.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&r.y));
    o[0] = a.x;
    o[1] = a.y;
    o[2] = b.x;
    o[3] = b.y;
  }
};
template <>
struct KvVec<__half, 2> {
  using Raw = uint32_t;
  static __device__ __forceinline__ Raw load(const __half* p) { return *reinterpret_cast<const uint32_t*>(p); }
  static __device__ __forceinline__ void cvt(const Raw& r, float (&o)[2]) {
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&r));
    o[0] = a.x;
    o[1] = a.y;
  }
};
template <>
struct KvVec<__half, 1> {
  using Raw = __half;
  static __device__ __forceinline__ Raw load(const __half* p) { return *p; }
  static __device__ __forceinline__ void cvt(const Raw& r, float (&o)[1]) { o[0] = __half2float(r); }
};

// fp8 e4m3 rows: 1, 2 or 4 bytes per lane, widened pairwise through fp16 (exact)
__device__ __forceinline__ float2 f8x2_to_float2(uint32_t b) {
  const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(b & 0xffffu), __NV_E4M3);
  return __half22float2(__half2(h));
}
template <>
struct KvVec<__nv_fp8_e4m3, 4> {
  using Raw = uint32_t;
  static __device__ __forceinline__ Raw load(const __nv_fp8_e4m3* p) { return *reinterpret_cast<const uint32_t*>(p); }
  static __device__ __forceinline__ void cvt(const Raw& r, float (&o)[4]) {
    const float2 a = f8x2_to_float2(r), b = f8x2_to_float2(r >> 16);
    o[0] = a.x;
    o[1] = a.y;
    o[2] = b.x;
    o[3] = b.y;
  }
};
template <>
struct KvVec<__nv_fp8_e4m3, 2> {
  using Raw = uint16_t;
  static __device__ __forceinline__ Raw load(const __nv_fp8_e4m3* p) { return *reinterpret_cast<const uint16_t*>(p); }
  static __device__ __forceinline__ void cvt(const Raw& r, float (&o)[2]) {
    const float2 a = f8x2_to_float2(r);
    o[0] = a.x;
    o[1] = a.y;
  }
};
template <>
struct KvVec<__nv_fp8_e4m3, 1> {
  using Raw = uint8_t;
  static __device__ __forceinline__ Raw load(const __nv_fp8_e4m3* p) { return *reinterpret_cast<const uint8_t*>(p); }
  static __device__ __forceinline__ void cvt(const Raw& r, float (&o)[1]) { o[0] = f8x2_to_float2(r).x; }
};

// after the loop lane holds the warp sum of v[lane >> (5 - log2 N)]
template <int N>
__device__ __forceinline__ float attn_reduce_scatter(float (&v)[N], int lane) {
#pragma unroll
  for (int n = N, o = 16; n > 1; n >>= 1, o >>= 1) {
    const bool upper = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < n / 2; i++) {
      const float send = upper ? v[i] : v[i + n / 2];
      const float keep = upper ? v[i + n / 2] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  constexpr int LOGN = N == 1 ? 0 : (N == 2 ? 1 : (N == 4 ? 2 : (N == 8 ? 3 : (N == 16 ? 4 : 5))));
  float r = v[0];
#pragma unroll
  for (int o = 16 >> LOGN; o >= 1; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
  return r;
}

// Two resident CTAs per SM (twice the loads in flight) where the registers
// allow it without spilling next to the next step's prefetched rows; the
// others keep the prefetch at one CTA per SM (a decoding row's grid has fewer
// CTAs than SMs anyway).
__host__ __device__ constexpr int attn_min_blocks(int HD, int G, bool half) {
  return G == 16 || (HD == 128 && G != 4) ? 1 : 2;
}
// registers of prefetched K (or V) rows a variant may hold: 16, except fp16
// rows at 4 query heads x 128 dimensions, which measured faster at two CTAs per
// SM without the prefetch (5.06 vs 4.54 TB/s over 64 rows of 32768 positions)
__host__ __device__ constexpr int attn_prefetch_regs(int HD, int G, bool half) {
  return HD == 128 && G == 4 && half ? 0 : 16;
}

// CL: the S splits of a (row, KV head) are one thread-block cluster and merge
// through distributed shared memory (S <= 8); else through the workspace.
// PG: the cache is paged (a.kv.pages), else contiguous per sequence slot.
template <int HD, int G, typename KT, bool CL, bool PG>
__global__ void __launch_bounds__(ATT_THREADS, attn_min_blocks(HD, G, sizeof(KT) < 4)) k_attn(const AttnArgs a) {
  constexpr int DPL = HD / 32, PS = 32 / G, GH = G * HD;
  using Vec = KvVec<KT, DPL>;
  using Raw = typename Vec::Raw;
  // prefetch the next step's K / V rows when they fit the variant's budget
  constexpr bool PF = PS * (((int)sizeof(Raw) + 3) / 4) <= attn_prefetch_regs(HD, G, sizeof(KT) == 2);
  constexpr unsigned FULL = 0xffffffffu;
  __shared__ float s_m[ATT_WARPS][G], s_l[ATT_WARPS][G];
  __shared__ __align__(16) float s_o[ATT_WARPS][GH];
  __shared__ float s_w[ATT_WARPS][G];  // merge weights exp(m - M) of the warps
  __shared__ float s_M[G], s_L[G];
  __shared__ __align__(16) float s_q[GH];  // this row's q for the G heads of the KV head
  __shared__ float s_part[2][ATT_MAX_SPLITS][G];  // the splits' maxima and sums (last arriver)
  __shared__ int s_last;
  __shared__ int s_pg[PG ? kAttnMaxPages : 1];  // (paged cache) the pages of this CTA's positions
  // grid.x = (row, KV head, split), a.S splits innermost
  const int split = (int)(blockIdx.x % a.S), kvh = (int)((blockIdx.x / a.S) % a.nkv);
  const int t = (int)(blockIdx.x / (a.S * a.nkv));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pdl_launch_dependents();
  pdl_wait();  // q and the cache rows of this step come from the previous kernels
  const RowInfo ri = a.rows[t];
  const int L = ri.len;
  // this row's splits: at most S, and at least two warp steps per warp each
  // (a short row takes few splits and a cheap merge; the rest exit here)
  constexpr int MINP = 2 * ATT_WARPS * PS;
  const int S = CL ? a.S : min(a.S, max(1, (L + MINP - 1) / MINP));  // (a cluster's CTAs all take part)
  if (split >= S) return;
  const int lo = (int)((int64_t)L * split / S), hi = (int)((int64_t)L * (split + 1) / S);
  const int wlo = lo + (int)((int64_t)(hi - lo) * warp / ATT_WARPS);
  const int whi = lo + (int)((int64_t)(hi - lo) * (warp + 1) / ATT_WARPS);
  // this lane's dimensions of position p's row at kb / vb + roff(p)
  const size_t base = (PG ? 0 : (size_t)ri.slot * a.kv.slot_stride) + kvh * a.kv.kvh_stride + lane * DPL;
  const KT* const kb = reinterpret_cast<const KT*>(a.kc) + base;
  const KT* const vb = reinterpret_cast<const KT*>(a.vc) + base;
  const int sh = a.kv.shift, pg0 = lo >> sh;
  auto roff = [&](int p) -> size_t {
    if constexpr (PG) return (size_t)s_pg[(p >> sh) - pg0] * a.kv.slot_stride + (size_t)(p & ((1 << sh) - 1)) * HD;
    else return (size_t)p * HD;
  };
  if constexpr (PG) {
    const int np = hi > lo ? ((hi - 1) >> sh) - pg0 + 1 : 0;  // <= kAttnMaxPages (checked by the host)
    for (int i = tid; i < np; i += ATT_THREADS) s_pg[i] = a.kv.pages[(size_t)ri.slot * a.kv.max_pages + pg0 + i];
    __syncthreads();
  }

  for (int e = tid; e < GH; e += ATT_THREADS) s_q[e] = a.q[(size_t)t * a.ldq + kvh * GH + e];
  float acc[G][DPL];
#pragma unroll
  for (int h = 0; h < G; h++)
#pragma unroll
    for (int d = 0; d < DPL; d++) acc[h][d] = 0.f;
  // this lane's DPL dimensions of head h's q
  auto q_of = [&](int h, float (&qh)[DPL]) {
    const float* src = s_q + h * HD + lane * DPL;
    if constexpr (DPL == 4) {
      const float4 v4 = *reinterpret_cast<const float4*>(src);
      qh[0] = v4.x;
      qh[DPL > 1 ? 1 : 0] = v4.y;
      qh[DPL > 2 ? 2 : 0] = v4.z;
      qh[DPL > 3 ? 3 : 0] = v4.w;
    } else {
#pragma unroll
      for (int d = 0; d < DPL; d++) qh[d] = src[d];
    }
  };
  // this lane's (head, position) after the reduce-scatter; its head's running
  // max / sum live in every lane of that head
  const int my_p = lane / G;
  float m_run = -INFINITY, l_run = 0.f;
  Raw kn[PF ? PS : 1], vn[PF ? PS : 1];
  auto load_step = [&](int p0, Raw (&kd)[PF ? PS : 1], Raw (&vd)[PF ? PS : 1]) {
#pragma unroll
    for (int i = 0; i < (PF ? PS : 1); i++) {
      const size_t o = roff(min(p0 + i, whi - 1));  // past the end: a valid row, masked below
      kd[i] = Vec::load(kb + o);
      vd[i] = Vec::load(vb + o);
    }
  };
  if (PF && wlo < whi) load_step(wlo, kn, vn);
  __syncthreads();  // s_q
  for (int p0 = wlo; p0 < whi; p0 += PS) {
    // this step's rows: K as floats for the scores, V kept raw until the
    // weighted sum converts it a position at a time
    float kr[PS][DPL];
    Raw vw[PS];
    if constexpr (PF) {
#pragma unroll
      for (int i = 0; i < PS; i++) {
        Vec::cvt(kn[i % (PF ? PS : 1)], kr[i]);
        vw[i] = vn[i % (PF ? PS : 1)];
      }
      if (p0 + PS < whi) load_step(p0 + PS, kn, vn);
    } else {
      Raw kw[PS];
#pragma unroll
      for (int i = 0; i < PS; i++) {
        const size_t o = roff(min(p0 + i, whi - 1));
        kw[i] = Vec::load(kb + o);
        vw[i] = Vec::load(vb + o);
      }
#pragma unroll
      for (int i = 0; i < PS; i++) Vec::cvt(kw[i], kr[i]);
    }
    float v[32];
#pragma unroll
    for (int h = 0; h < G; h++) {
      float qh[DPL];
      q_of(h, qh);
#pragma unroll
      for (int i = 0; i < PS; i++) {
        float s = 0.f;
#pragma unroll
        for (int d = 0; d < DPL; d++) s = fmaf(qh[d], kr[i][d], s);
        v[i * G + h] = s;
      }
    }
    const float sc = attn_reduce_scatter<32>(v, lane) * a.scale;
    const float s = p0 + my_p < whi ? sc : -INFINITY;
    float mx = s;
#pragma unroll
    for (int o = G; o < 32; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, o));
    const float m_new = fmaxf(m_run, mx);  // finite: position p0 is always valid
    const float p = s == -INFINITY ? 0.f : expf(s - m_new);
    const float alpha = m_run == -INFINITY ? 0.f : expf(m_run - m_new);
    float ps = p;
#pragma unroll
    for (int o = G; o < 32; o <<= 1) ps += __shfl_xor_sync(FULL, ps, o);
    l_run = l_run * alpha + ps;
    m_run = m_new;
#pragma unroll
    for (int h = 0; h < G; h++) {
      const float al = __shfl_sync(FULL, alpha, h);
#pragma unroll
      for (int d = 0; d < DPL; d++) acc[h][d] *= al;
    }
#pragma unroll
    for (int i = 0; i < PS; i++) {
      float vr[DPL];
      Vec::cvt(vw[i], vr);
#pragma unroll
      for (int h = 0; h < G; h++) {
        const float w = __shfl_sync(FULL, p, i * G + h);
#pragma unroll
        for (int d = 0; d < DPL; d++) acc[h][d] = fmaf(w, vr[d], acc[h][d]);
      }
    }
  }
  // merge the warps: the CTA's partial is the output relative to its
  // per-head max M, with the sum L
  if (lane < G) {
    s_m[warp][lane] = m_run;
    s_l[warp][lane] = l_run;
  }
#pragma unroll
  for (int h = 0; h < G; h++)
#pragma unroll
    for (int d = 0; d < DPL; d++) s_o[warp][h * HD + lane * DPL + d] = acc[h][d];
  __syncthreads();
  if (tid < G) {
    float M = -INFINITY;
    for (int w = 0; w < ATT_WARPS; w++) M = fmaxf(M, s_m[w][tid]);
    float Lsum = 0.f;
    for (int w = 0; w < ATT_WARPS; w++) {
      const float f = s_m[w][tid] == -INFINITY ? 0.f : expf(s_m[w][tid] - M);
      s_w[w][tid] = f;
      Lsum += s_l[w][tid] * f;
    }
    s_M[tid] = M;
    s_L[tid] = Lsum;
  }
  __syncthreads();
  const size_t pbase = ((size_t)t * a.nkv + kvh) * a.S;  // this (row, KV head)'s first partial
  float* const wp = a.ws + (pbase + split) * a.pstride;
  for (int e = tid; e < GH; e += ATT_THREADS) {
    const int h = e / HD;
    float o = 0.f;
    for (int w = 0; w < ATT_WARPS; w++) o = fmaf(s_o[w][e], s_w[w][h], o);
    if (S == 1) a.out[(size_t)t * a.ldo + (kvh * G + h) * HD + e % HD] = s_L[h] > 0.f ? o / s_L[h] : 0.f;
    else if (CL) s_o[0][e] = o;  // (element e is read and rewritten by this thread only)
    else wp[e] = o;
  }
  if (S == 1) return;
  if constexpr (CL) {
    // after the barrier, split r finalises outputs [r GH / S, (r + 1) GH / S)
    // from every split's partial, read from the others' shared memory in
    // split order; the second barrier keeps the partials alive until then
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    for (int e = GH * split / S + tid; e < GH * (split + 1) / S; e += ATT_THREADS) {
      const int h = e / HD;
      float M = -INFINITY;
      for (int c = 0; c < S; c++) M = fmaxf(M, *cluster.map_shared_rank(&s_M[h], c));
      float Lsum = 0.f, o = 0.f;
      for (int c = 0; c < S; c++) {
        const float mc = *cluster.map_shared_rank(&s_M[h], c);
        const float f = mc == -INFINITY ? 0.f : expf(mc - M);
        Lsum += *cluster.map_shared_rank(&s_L[h], c) * f;
        o = fmaf(*cluster.map_shared_rank(&s_o[0][e], c), f, o);
      }
      a.out[(size_t)t * a.ldo + (kvh * G + h) * HD + e % HD] = Lsum > 0.f ? o / Lsum : 0.f;
    }
    cluster.sync();
    return;
  }
  if (tid < G) {
    wp[GH + tid] = s_M[tid];
    wp[GH + G + tid] = s_L[tid];
  }
  // publish the partial; the last of the S CTAs to arrive merges
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = atom_add_acq_rel(a.cnt + (size_t)t * a.nkv + kvh, 1) == S - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const float* w0 = a.ws + pbase * a.pstride;
  for (int i = tid; i < 2 * S * G; i += ATT_THREADS) {
    const int c = i / (2 * G), r = i % (2 * G);
    s_part[r / G][c][r % G] = __ldcg(w0 + (size_t)c * a.pstride + GH + r);
  }
  __syncthreads();
  if (tid < G) {
    float M = -INFINITY;
    for (int c = 0; c < S; c++) M = fmaxf(M, s_part[0][c][tid]);
    float Lsum = 0.f;
    for (int c = 0; c < S; c++) {
      const float mc = s_part[0][c][tid];
      const float f = mc == -INFINITY ? 0.f : expf(mc - M);
      Lsum += s_part[1][c][tid] * f;
      s_part[0][c][tid] = f;  // (column tid is read and rewritten by this thread only)
    }
    s_L[tid] = Lsum;
  }
  __syncthreads();
  // this thread's EPT output elements, CB splits at a time: 32 loads in flight
  constexpr int EPT = (GH + ATT_THREADS - 1) / ATT_THREADS, CB = 32 / EPT > 0 ? 32 / EPT : 1;
  float o[EPT];
#pragma unroll
  for (int i = 0; i < EPT; i++) o[i] = 0.f;
  for (int c0 = 0; c0 < S; c0 += CB) {
    float pv[CB][EPT];
#pragma unroll
    for (int j = 0; j < CB; j++)
#pragma unroll
      for (int i = 0; i < EPT; i++) {
        const int e = tid + i * ATT_THREADS;
        pv[j][i] = c0 + j < S && e < GH ? __ldcg(w0 + (size_t)(c0 + j) * a.pstride + e) : 0.f;
      }
#pragma unroll
    for (int j = 0; j < CB; j++)
#pragma unroll
      for (int i = 0; i < EPT; i++) {
        const int e = tid + i * ATT_THREADS;
        if (c0 + j < S && e < GH) o[i] = fmaf(pv[j][i], s_part[0][c0 + j][e / HD], o[i]);
      }
  }
#pragma unroll
  for (int i = 0; i < EPT; i++) {
    const int e = tid + i * ATT_THREADS, h = e / HD;
    if (e < GH) a.out[(size_t)t * a.ldo + (kvh * G + h) * HD + e % HD] = s_L[h] > 0.f ? o[i] / s_L[h] : 0.f;
  }
  if (tid == 0) a.cnt[(size_t)t * a.nkv + kvh] = 0;  // ready for the next launch
}

// ---------------------------------------------------------------- host side
using AttnLaunch = cudaError_t (*)(const AttnArgs&, dim3, cudaStream_t);
struct AttnKernel {
  const void* fn = nullptr;
  AttnLaunch launch = nullptr;
};

template <int HD, int G, typename KT, bool PG>
static cudaError_t attn_launch_pg(const AttnArgs& a, dim3 grid, cudaStream_t s) {
  if (a.ws == nullptr && a.S > 1)  // cluster merge
    return launch_pdl_cluster(k_attn<HD, G, KT, true, PG>, grid, dim3(ATT_THREADS), 0, a.S, s, a);
  return launch_pdl(k_attn<HD, G, KT, false, PG>, grid, dim3(ATT_THREADS), 0, s, a);
}
template <int HD, int G, typename KT>
static cudaError_t attn_launch_t(const AttnArgs& a, dim3 grid, cudaStream_t s) {
  return a.kv.pages ? attn_launch_pg<HD, G, KT, true>(a, grid, s) : attn_launch_pg<HD, G, KT, false>(a, grid, s);
}
template <int HD, int G, typename KT>
static AttnKernel attn_k() {
  return AttnKernel{(const void*)k_attn<HD, G, KT, false, false>, attn_launch_t<HD, G, KT>};
}
template <int HD, typename KT>
static bool attn_kernel_hd(int G, AttnKernel* k) {
  switch (G) {
    case 1: *k = attn_k<HD, 1, KT>(); return true;
    case 2: *k = attn_k<HD, 2, KT>(); return true;
    case 4: *k = attn_k<HD, 4, KT>(); return true;
    case 8: *k = attn_k<HD, 8, KT>(); return true;
    case 16:
      if (HD > 64) return false;  // 16 x 128 accumulators do not fit a lane
      *k = attn_k<(HD > 64 ? 64 : HD), 16, KT>();
      return true;
    default: return false;
  }
}
template <typename KT>
static bool attn_kernel_kt(int hd, int G, AttnKernel* k) {
  switch (hd) {
    case 32: return attn_kernel_hd<32, KT>(G, k);
    case 64: return attn_kernel_hd<64, KT>(G, k);
    case 128: return attn_kernel_hd<128, KT>(G, k);
    default: return false;
  }
}
static bool attn_kernel(int hd, int G, int kv_type, AttnKernel* k) {
  if (kv_type == KV_F16) return attn_kernel_kt<__half>(hd, G, k);
  if (kv_type == KV_F8) return attn_kernel_kt<__nv_fp8_e4m3>(hd, G, k);
  return attn_kernel_kt<float>(hd, G, k);
}

// resident CTAs per SM of a variant (looked up once per variant)
static int attn_occupancy(int hd, int G, int kv_type) {
  static std::atomic<int> cache[3][5][3];
  const int hi = hd == 32 ? 0 : hd == 64 ? 1 : 2, gi = G == 1 ? 0 : G == 2 ? 1 : G == 4 ? 2 : G == 8 ? 3 : 4;
  std::atomic<int>& c = cache[hi][gi][kv_type == KV_F16 ? 1 : (kv_type == KV_F8 ? 2 : 0)];
  int o = c.load(std::memory_order_relaxed);
  if (o > 0) return o;
  AttnKernel k;
  o = 1;
  if (attn_kernel(hd, G, kv_type, &k) &&
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, k.fn, ATT_THREADS, 0) != cudaSuccess) {
    cudaGetLastError();
    o = 1;
  }
  o = std::max(1, o);
  c.store(o, std::memory_order_relaxed);
  return o;
}

AttnPlan attn_plan(int T, int nH, int nKV, int hd, int max_ctx, int kv_type, size_t ws_cap_floats) {
  AttnPlan p;
  if (T <= 0 || nKV <= 0 || nH % nKV != 0) return p;
  const int G = nH / nKV, PS = 32 / std::max(1, std::min(G, 32));
  // splits so that the grid fills every SM's resident CTA slots in one wave
  // (never a second, mostly idle one), each split at least one warp step per
  // warp of the longest row
  const int64_t rows_kv = (int64_t)T * nKV;
  const int64_t target = (int64_t)attn_occupancy(hd, G, kv_type) * num_sms();
  int S = (int)std::max<int64_t>(1, target / rows_kv);
  S = std::min(S, std::max(1, (max_ctx + ATT_WARPS * PS - 1) / (ATT_WARPS * PS)));
  S = std::min(S, ATT_MAX_SPLITS);
  // Up to 8 splits, and any split count over caches of <= kAttnClusterCtx
  // positions, merge within a cluster: no global round trip, which the decode
  // chain's short rows feel most.  More splits over longer caches go through
  // the workspace.
  if (S <= 8 || max_ctx <= kAttnClusterCtx) {
    p.splits = std::min(S, 8);
    p.cluster = p.splits > 1;
    return p;
  }
  const size_t per = (size_t)rows_kv * attn_pstride(G, hd);
  while (S > 8 && per * S > ws_cap_floats) S--;
  if (per * S > ws_cap_floats) S = 8;  // no room: the cluster merge
  p.splits = S;
  p.cluster = S <= 8;
  p.ws_floats = p.cluster ? 0 : per * S;
  p.cnt_ints = p.cluster ? 0 : (size_t)rows_kv;
  return p;
}

int attention(const float* q, int ldq, const void* kc, const void* vc, int kv_type, const KvMap& kv,
              const RowInfo* rows, int T, int nH, int nKV, int hd, const AttnPlan& plan, float* out, int ldo,
              float* ws, int* cnt, cudaStream_t s) {
  if (T <= 0) return TN_OK;
  TN_REQUIRE(nKV > 0 && nH % nKV == 0, TN_EUNSUPPORTED, "attention: n_heads %% n_kv_heads != 0");
  TN_REQUIRE(plan.splits >= 1 && plan.splits <= ATT_MAX_SPLITS, TN_EINVAL, "attention: %d splits", plan.splits);
  TN_REQUIRE(plan.splits == 1 || plan.cluster || (ws && cnt), TN_EINVAL, "attention: split workspace missing");
  TN_REQUIRE(!plan.cluster || plan.splits <= 8, TN_EINVAL, "attention: cluster of %d splits", plan.splits);
  if (plan.cluster || plan.splits == 1) {
    ws = nullptr;  // (selects the cluster merge)
    cnt = nullptr;
  }
  const int G = nH / nKV;
  AttnKernel k;
  if (!attn_kernel(hd, G, kv_type, &k)) {
    set_error("attention: %d query heads per KV head with head_dim %d unsupported", G, hd);
    return TN_EUNSUPPORTED;
  }
  TN_REQUIRE(!kv.pages || (kv.shift >= 0 && kv.shift < 30), TN_EINVAL, "attention: page shift %d", kv.shift);
  const AttnArgs a{q,   ldq, kc,  vc,         kv, rows, plan.splits, nKV, (float)(1.0 / sqrt((double)hd)),
                   out, ldo, ws, cnt, attn_pstride(G, hd)};
  const dim3 grid((unsigned)((int64_t)plan.splits * nKV * T));
  TN_CHECK_CUDA(k.launch(a, grid, s));
  return TN_OK;
}

}  // namespace tn
