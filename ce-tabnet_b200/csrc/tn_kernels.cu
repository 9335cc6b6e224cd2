// tn_kernels.cu -- sm_100a kernels of the stage engine.
//
// Math follows the reference CPU path (web/inference-worker.js:509-583) in
// f32 storage with f32 accumulation (the reference accumulates in double;
// parity is a 1e-3 max-relative bound on hidden states, greedy tokens exact).
// The transcendental pieces that the reference evaluates in double (RMS, RoPE
// rotation, softmax normaliser of the sampler) are evaluated in double here too.
#include <cfloat>

#include "tn_kernels.cuh"

namespace tn {

int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  }
  return n;
}

// ---------------------------------------------------------------- loads
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// ================================================================ repack
// Reference block at element index i of a packed tensor (blocks over the flat
// tensor, web/inference-worker.js:107-124): exact f32 value.
__device__ __forceinline__ float packed_elem(const uint8_t* src, int quant, uint64_t i) {
  if (quant == TN_QUANT_F32) {
    const uint8_t* p = src + i * 4;
    return u2f((uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24));
  }
  if (quant == TN_QUANT_F16) {
    const uint8_t* p = src + i * 2;
    return f16_to_f32((uint16_t)(p[0] | (p[1] << 8)));
  }
  const uint64_t b = i >> 5, j = i & 31;
  if (quant == TN_QUANT_Q8_0) {
    const uint8_t* blk = src + b * 34;
    const float d = f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
    return (float)(int8_t)blk[2 + j] * d;
  }
  const uint8_t* blk = src + b * 18;
  const float d = f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
  const uint8_t byte = blk[2 + (j >> 1)];
  const int nib = (j & 1) ? (byte >> 4) : (byte & 15);
  return (float)(nib - 8) * d;
}

// Destination row of source row r: dst_off + r * dst_stride, or, for a
// negative stride, the RoPE pair-interleaved order of heads of -dst_stride
// rows: within a head, rows i and i + hd/2 (a rotation pair of
// web/inference-worker.js:535-537) land next to each other at 2i and 2i + 1,
// so one epilogue thread sees both halves of every pair.
__host__ __device__ __forceinline__ uint64_t dst_row(uint64_t r, int dst_off, int dst_stride) {
  if (dst_stride > 0) return (uint64_t)dst_off + r * (uint64_t)dst_stride;
  const uint64_t hd = (uint64_t)(-dst_stride), half = hd / 2, h = r / hd, j = r % hd;
  return (uint64_t)dst_off + h * hd + (j < half ? 2 * j : 2 * (j - half) + 1);
}

// Source row that dst_row maps onto destination row d, or -1 if none of this
// repack's rows lands there.
__device__ __forceinline__ int64_t src_row_of(int64_t d, int dst_off, int dst_stride, int src_rows) {
  const int64_t rel = d - dst_off;
  if (rel < 0) return -1;
  int64_t r;
  if (dst_stride > 0) {
    if (rel % dst_stride) return -1;
    r = rel / dst_stride;
  } else {
    const int64_t hd = -dst_stride, half = hd / 2, h = rel / hd, j = rel % hd;
    r = h * hd + ((j & 1) ? half + (j >> 1) : (j >> 1));
  }
  return r < src_rows ? r : -1;
}

// Block-aligned q4_0 / q8_0 source into the fragment-ordered records: one
// thread per (tile, g, pair) writes the 4 lane slots 4g .. 4g + 3 and the
// scale words of rows g and g + 8.  Rows of the tile that another repack call
// owns keep their bytes (read-modify-write; calls are stream ordered).
template <int KIND>
__global__ void k_repack_tile(const uint8_t* __restrict__ src, int src_rows, int nb, int pairs, int tiles,
                              int dst_off, int dst_stride, uint8_t* __restrict__ data) {
  constexpr int BB = KIND == MK_Q4 ? 18 : 34;
  constexpr int AB = tile_a_bytes(KIND), REC = tile_rec_bytes(KIND), LB = AB / 32;
  const uint64_t total = (uint64_t)tiles * 8 * pairs;
  for (uint64_t k = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; k < total;
       k += (uint64_t)gridDim.x * blockDim.x) {
    const int p = (int)(k % pairs);
    const uint64_t tg = k / pairs;
    const int g = (int)(tg & 7);
    const int64_t t = (int64_t)(tg >> 3);
    const int64_t rs[2] = {src_row_of(t * 16 + g, dst_off, dst_stride, src_rows),
                           src_row_of(t * 16 + g + 8, dst_off, dst_stride, src_rows)};
    if (rs[0] < 0 && rs[1] < 0) continue;
    const uint8_t* blk[2][2];  // [u = row g / g + 8][q]
#pragma unroll
    for (int u = 0; u < 2; u++)
#pragma unroll
      for (int q = 0; q < 2; q++)
        blk[u][q] = (rs[u] >= 0 && 2 * p + q < nb) ? src + ((size_t)rs[u] * nb + 2 * p + q) * BB : nullptr;
    uint8_t* rec = data + ((size_t)t * pairs + p) * REC;
#pragma unroll
    for (int c = 0; c < 4; c++) {
      uint8_t* lane = rec + (4 * g + c) * LB;
#pragma unroll
      for (int h = 0; h < 2; h++)
#pragma unroll
        for (int q = 0; q < 2; q++)
#pragma unroll
          for (int i = 0; i < 4; i++) {
            const int e = 16 * h + 4 * c + i;
            if (KIND == MK_Q4) {
              uint8_t* byte = lane + (2 * h + q) * 4 + i;
              uint8_t v = *byte;
              if (blk[0][q]) {
                const uint8_t sb = blk[0][q][2 + (e >> 1)];
                v = (uint8_t)((v & 0x0F) | ((((e & 1) ? sb >> 4 : sb & 15) ^ 8) << 4));
              }
              if (blk[1][q]) {
                const uint8_t sb = blk[1][q][2 + (e >> 1)];
                v = (uint8_t)((v & 0xF0) | (((e & 1) ? sb >> 4 : sb & 15) ^ 8));
              }
              *byte = v;
            } else {
#pragma unroll
              for (int u = 0; u < 2; u++)
                if (blk[u][q]) lane[(4 * h + 2 * q + u) * 4 + i] = blk[u][q][2 + e];
            }
          }
    }
    uint16_t* sc = reinterpret_cast<uint16_t*>(rec + AB);
#pragma unroll
    for (int q = 0; q < 2; q++)
#pragma unroll
      for (int u = 0; u < 2; u++)
        if (blk[u][q]) sc[(2 * g + q) * 2 + u] = (uint16_t)(blk[u][q][0] | (blk[u][q][1] << 8));
  }
}

// any source format into an MK_F32 / MK_F16 matrix (exact values)
__global__ void k_repack_plain(const uint8_t* __restrict__ src, int quant, int src_rows, int cols,
                               int cols_pad, int dst_off, int dst_stride, int kind,
                               uint8_t* __restrict__ data) {
  const uint64_t total = (uint64_t)src_rows * cols;
  for (uint64_t k = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; k < total;
       k += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t r = k / cols, c = k % cols;
    const uint64_t dr = dst_row(r, dst_off, dst_stride);
    if (kind == MK_F16) {
      const uint8_t* p = src + k * 2;
      ((uint16_t*)data)[dr * cols_pad + c] = (uint16_t)(p[0] | (p[1] << 8));
    } else {
      ((float*)data)[dr * cols_pad + c] = packed_elem(src, quant, k);
    }
  }
}

static void mv_prepare(Matrix* m);

int matrix_alloc(Matrix* m, int src_quant, int rows, int cols, cudaStream_t s, bool own_ws) {
  TN_REQUIRE(rows > 0 && cols > 0, TN_EINVAL, "matrix: bad shape %d x %d", rows, cols);
  TN_REQUIRE(quant_bytes(1, src_quant) != 0, TN_EUNSUPPORTED, "unsupported quant %d", src_quant);
  m->rows = rows;
  m->cols = cols;
  m->rows_pad = (rows + 15) & ~15;
  m->cols_pad = (cols + 31) & ~31;
  m->nb = m->cols_pad / 32;
  const bool aligned = (cols % 32) == 0;
  if (src_quant == TN_QUANT_Q4_0 && aligned) m->kind = MK_Q4;
  else if (src_quant == TN_QUANT_Q8_0 && aligned) m->kind = MK_Q8;
  else if (src_quant == TN_QUANT_F16) m->kind = MK_F16;
  else m->kind = MK_F32;
  size_t dbytes;
  if (m->kind == MK_Q4 || m->kind == MK_Q8) {
    m->tiles = m->rows_pad / 16;
    m->pairs = (m->nb + 1) / 2;
    dbytes = (size_t)m->tiles * m->pairs * tile_rec_bytes(m->kind);
  } else {
    dbytes = (size_t)m->rows_pad * m->nb * kind_block_bytes(m->kind);
  }
  TN_CHECK_CUDA(cudaMalloc(&m->data, dbytes));
  // zero padding rows/columns on the stream the repack kernels will use
  TN_CHECK_CUDA(cudaMemsetAsync(m->data, 0, dbytes, s));
  m->bytes = dbytes;
  num_sms();
  if (m->kind == MK_Q4 || m->kind == MK_Q8) {
    const int rc = mm_prepare(m);
    if (rc != TN_OK) return rc;
    m->has_wmap = gemm_encode_maps(m);  // without them the GEMM is not used
    m->ws_owned = own_ws;
    if (m->ws_floats && own_ws) {
      const size_t wsb = m->ws_floats * sizeof(float);
      TN_CHECK_CUDA(cudaMalloc(&m->ws, wsb));
      TN_CHECK_CUDA(cudaMemsetAsync(m->ws, 0, wsb, s));
      TN_CHECK_CUDA(cudaMalloc(&m->cnt, m->cnt_ints * sizeof(int)));
      TN_CHECK_CUDA(cudaMemsetAsync(m->cnt, 0, m->cnt_ints * sizeof(int), s));
      m->bytes += wsb + m->cnt_ints * sizeof(int);
    }
  } else {
    mv_prepare(m);
  }
  return TN_OK;
}

int matrix_repack(Matrix* m, const uint8_t* d_src, int src_quant, int src_rows, int dst_off,
                  int dst_stride, cudaStream_t s) {
  TN_REQUIRE(dst_stride != 0 && (dst_stride > 0 || src_rows % (-dst_stride) == 0), TN_EINVAL,
             "matrix_repack: bad row stride %d", dst_stride);
  TN_REQUIRE(dst_off + (int64_t)(src_rows - 1) * (dst_stride > 0 ? dst_stride : 1) < m->rows, TN_EINVAL,
             "matrix_repack: rows out of range");
  if (m->kind == MK_Q4 || m->kind == MK_Q8) {
    const int64_t work = (int64_t)m->tiles * 8 * m->pairs;
    const int grid = (int)std::min<int64_t>(148 * 32, std::max<int64_t>(1, (work + 255) / 256));
    if (m->kind == MK_Q4)
      k_repack_tile<MK_Q4><<<grid, 256, 0, s>>>(d_src, src_rows, m->nb, m->pairs, m->tiles, dst_off, dst_stride,
                                                m->data);
    else
      k_repack_tile<MK_Q8><<<grid, 256, 0, s>>>(d_src, src_rows, m->nb, m->pairs, m->tiles, dst_off, dst_stride,
                                                m->data);
  } else {
    const int grid = std::min(148 * 32, (int)std::max<int64_t>(1, ((int64_t)src_rows * m->nb + 255) / 256));
    k_repack_plain<<<grid, 256, 0, s>>>(d_src, src_quant, src_rows, m->cols, m->cols_pad, dst_off,
                                        dst_stride, m->kind, m->data);
  }
  TN_CHECK_LAUNCH();
  return TN_OK;
}

void matrix_free(Matrix* m) {
  if (m->data) cudaFree(m->data);
  if (m->ws_owned) {
    if (m->ws) cudaFree(m->ws);
    if (m->cnt) cudaFree(m->cnt);
  }
  m->data = nullptr;
  m->ws = nullptr;
  m->cnt = nullptr;
  m->bytes = 0;
}

void matrix_reset_counters(const Matrix& m, cudaStream_t s) {
  if (m.cnt) cudaMemsetAsync(m.cnt, 0, m.cnt_ints * sizeof(int), s);
  if (m.ws) cudaMemsetAsync(m.ws, 0, m.ws_floats * sizeof(float), s);
}

// value of element (r, c) of a repacked matrix
__device__ __forceinline__ float mat_elem(int kind, const uint8_t* data, int nb, int cols_pad, uint64_t r,
                                          int c) {
  if (kind == MK_F32) return ((const float*)data)[r * cols_pad + c];
  if (kind == MK_F16) return f16_to_f32(((const uint16_t*)data)[r * cols_pad + c]);
  const int pairs = (nb + 1) >> 1, rr = (int)(r & 15), g = rr & 7, u = rr >> 3;
  const int b = c >> 5, e = c & 31, p = b >> 1, q = b & 1, h = e >> 4, cc = (e & 15) >> 2, i = e & 3;
  const int ab = kind == MK_Q4 ? 512 : 1024;
  const uint8_t* rec = data + ((r >> 4) * pairs + p) * (uint64_t)(ab + 64);
  const float d = f16_to_f32(reinterpret_cast<const uint16_t*>(rec + ab)[(2 * g + q) * 2 + u]);
  if (kind == MK_Q8) return (float)(int8_t)rec[(4 * g + cc) * 32 + (4 * h + 2 * q + u) * 4 + i] * d;
  const uint8_t byte = rec[(4 * g + cc) * 16 + (2 * h + q) * 4 + i];
  const int s = u ? (byte & 15) : (byte >> 4);
  return (float)((s ^ 8) - 8) * d;
}

__global__ void k_dequant(int kind, const uint8_t* data, int rows, int cols, int nb, int cols_pad, float* out) {
  const uint64_t total = (uint64_t)rows * cols;
  for (uint64_t k = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; k < total;
       k += (uint64_t)gridDim.x * blockDim.x)
    out[k] = mat_elem(kind, data, nb, cols_pad, k / cols, (int)(k % cols));
}

int matrix_dequant(const Matrix& m, float* out, cudaStream_t s) {
  const int grid = std::min(148 * 32, (int)std::max<int64_t>(1, ((int64_t)m.rows * m.cols + 255) / 256));
  k_dequant<<<grid, 256, 0, s>>>(m.kind, m.data, m.rows, m.cols, m.nb, m.cols_pad, out);
  TN_CHECK_LAUNCH();
  return TN_OK;
}

// ================================================================ matvec (f16 / f32)
// CUDA-core matvec of the row-major kinds (f16 / f32 tensors, and q4_0 /
// q8_0 tensors whose rows straddle blocks, held dequantised).  Each thread of
// a CTA owns NBT 32-wide block columns of K and keeps x for them in
// registers; the CTA walks a contiguous range of 8-row groups, streaming
// weights with 128-bit loads, and reduces each group's 8 x TT partial dot
// products with a warp reduce-scatter plus one shared-memory pass.
template <int KIND, int NBT>
struct MvCfg {
  static constexpr int W = kind_block_bytes(KIND) / 4;  // 32-bit words per block
  static constexpr int RG0 = 32 / (W * NBT);
  static constexpr int RG = RG0 < 1 ? 1 : (RG0 > 8 ? 8 : RG0);  // rows loaded per sub-step
};

template <int N>
__device__ __forceinline__ float warp_reduce_scatter(float (&v)[N], int lane) {
  // after the loop lane holds the warp sum of v[lane >> (5 - log2 N)]
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

template <int KIND, int TT, int NBT>
__global__ void __launch_bounds__(512) k_matvec(const uint8_t* __restrict__ data, int rows, int rows_pad,
                                                int cols, int nb, int T, const float* __restrict__ x,
                                                int ldx, float* __restrict__ y, int ldy, int mode) {
  static_assert(KIND == MK_F16 || KIND == MK_F32, "row-major kinds only");
  using C = MvCfg<KIND, NBT>;
  constexpr int W = C::W, RG = C::RG, N = 8 * TT;
  constexpr int BB = kind_block_bytes(KIND);
  __shared__ float red[2][16][N];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  const int G = rows_pad >> 3;
  const int g0 = (int)((int64_t)G * blockIdx.x / gridDim.x);
  const int g1 = (int)((int64_t)G * (blockIdx.x + 1) / gridDim.x);
  int buf = 0;

  for (int t0 = 0; t0 < T; t0 += TT) {
    float xr[TT][NBT][32];
#pragma unroll
    for (int tt = 0; tt < TT; tt++)
#pragma unroll
      for (int j = 0; j < NBT; j++) {
        const int b = tid + j * blockDim.x;
        const bool ok = b < nb && t0 + tt < T;
#pragma unroll
        for (int e = 0; e < 32; e += 4) {
          float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
          const int c = b * 32 + e;
          if (ok) {
            const float* px = x + (size_t)(t0 + tt) * ldx + c;
            if (c + 3 < cols && (reinterpret_cast<uintptr_t>(px) & 15) == 0)
              v = *reinterpret_cast<const float4*>(px);
            else {
              v.x = c < cols ? px[0] : 0.f;
              v.y = c + 1 < cols ? px[1] : 0.f;
              v.z = c + 2 < cols ? px[2] : 0.f;
              v.w = c + 3 < cols ? px[3] : 0.f;
            }
          }
          xr[tt][j][e] = v.x;
          xr[tt][j][e + 1] = v.y;
          xr[tt][j][e + 2] = v.z;
          xr[tt][j][e + 3] = v.w;
        }
      }

    for (int g = g0; g < g1; g++) {
      float acc[8][TT];
#pragma unroll
      for (int i = 0; i < 8; i++)
#pragma unroll
        for (int tt = 0; tt < TT; tt++) acc[i][tt] = 0.f;

#pragma unroll
      for (int rs = 0; rs < 8; rs += RG) {
#pragma unroll
        for (int j = 0; j < NBT; j++) {
          const int b = tid + j * blockDim.x;
          if (b < nb) {
            uint32_t w[RG][W];
#pragma unroll
            for (int i = 0; i < RG; i++) {
              const uint8_t* p = data + ((size_t)(g * 8 + rs + i) * nb + b) * BB;
#pragma unroll
              for (int v = 0; v < W / 4; v++) {
                const uint4 q = ld_stream(p + 16 * v);
                w[i][4 * v] = q.x;
                w[i][4 * v + 1] = q.y;
                w[i][4 * v + 2] = q.z;
                w[i][4 * v + 3] = q.w;
              }
            }
#pragma unroll
            for (int i = 0; i < RG; i++) {
#pragma unroll
              for (int tt = 0; tt < TT; tt++) {
                float s = 0.f;
                if (KIND == MK_F16) {
#pragma unroll
                  for (int k = 0; k < 16; k++) {
                    const __half2 h2 = *reinterpret_cast<const __half2*>(&w[i][k]);
                    const float2 f2 = __half22float2(h2);
                    s = fmaf(f2.x, xr[tt][j][2 * k], s);
                    s = fmaf(f2.y, xr[tt][j][2 * k + 1], s);
                  }
                  acc[rs + i][tt] += s;
                } else {
#pragma unroll
                  for (int k = 0; k < 32; k++) s = fmaf(__uint_as_float(w[i][k]), xr[tt][j][k], s);
                  acc[rs + i][tt] += s;
                }
              }
            }
          }
        }
      }

      float v[N];
#pragma unroll
      for (int i = 0; i < 8; i++)
#pragma unroll
        for (int tt = 0; tt < TT; tt++) v[i * TT + tt] = acc[i][tt];
      const float r = warp_reduce_scatter<N>(v, lane);
      constexpr int SH = 5 - (N == 8 ? 3 : 4);
      if ((lane & ((1 << SH) - 1)) == 0) red[buf][warp][lane >> SH] = r;
      __syncthreads();
      if (mode == EPI_SWIGLU) {
        if (tid < 4 * TT) {
          const int pr = tid / TT, tt = tid % TT, t = t0 + tt;
          float sg = 0.f, su = 0.f;
          for (int w2 = 0; w2 < nwarps; w2++) {
            sg += red[buf][w2][(2 * pr) * TT + tt];
            su += red[buf][w2][(2 * pr + 1) * TT + tt];
          }
          const int row = g * 8 + 2 * pr;
          if (row + 1 < rows && t < T) y[(size_t)t * ldy + (row >> 1)] = (sg / (1.0f + expf(-sg))) * su;
        }
      } else if (tid < N) {
        const int i = tid / TT, tt = tid % TT, t = t0 + tt, row = g * 8 + i;
        float s = 0.f;
        for (int w2 = 0; w2 < nwarps; w2++) s += red[buf][w2][tid];
        if (row < rows && t < T) {
          float* py = y + (size_t)t * ldy + row;
          if (mode == EPI_RESID) *py = *py + s;
          else *py = s;
        }
      }
      buf ^= 1;
    }
  }
}

template <int KIND, int TT, int NBT>
static int mv_threads(const Matrix& m) {
  return ((m.nb + NBT - 1) / NBT + 31) & ~31;
}

template <int KIND, int TT, int NBT>
static int mv_occupancy(const Matrix& m) {
  int o = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, k_matvec<KIND, TT, NBT>, mv_threads<KIND, TT, NBT>(m), 0) !=
          cudaSuccess ||
      o <= 0)
    o = 1;
  return o;
}

template <int KIND, int TT, int NBT>
static int launch_mv(const Matrix& m, int T, const float* x, int ldx, float* y, int ldy, int mode,
                     cudaStream_t s) {
  const int G = m.rows_pad / 8;
  const int occ = m.occ[TT - 1] > 0 ? m.occ[TT - 1] : 1;
  const int grid = std::max(1, std::min(G, occ * num_sms()));
  k_matvec<KIND, TT, NBT><<<grid, mv_threads<KIND, TT, NBT>(m), 0, s>>>(m.data, m.rows, m.rows_pad, m.cols, m.nb,
                                                                          T, x, ldx, y, ldy, mode);
  TN_CHECK_LAUNCH();
  return TN_OK;
}

// occupancy of the launch shapes a matrix will use, queried once at allocation
// (never inside a CUDA graph capture)
template <int KIND>
static void mv_prepare_kind(Matrix* m) {
  if (m->nb <= 512) {
    m->occ[0] = mv_occupancy<KIND, 1, 1>(*m);
    m->occ[1] = mv_occupancy<KIND, 2, 1>(*m);
  } else {
    m->occ[0] = m->occ[1] = mv_occupancy<KIND, 1, 2>(*m);
  }
}

static void mv_prepare(Matrix* m) {
  if (m->kind == MK_F16) mv_prepare_kind<MK_F16>(m);
  else mv_prepare_kind<MK_F32>(m);
}

template <int KIND>
static int matvec_kind(const Matrix& m, int T, const float* x, int ldx, float* y, int ldy, int mode,
                       cudaStream_t s) {
  if (m.nb <= 512) {
    if (T >= 2) return launch_mv<KIND, 2, 1>(m, T, x, ldx, y, ldy, mode, s);
    return launch_mv<KIND, 1, 1>(m, T, x, ldx, y, ldy, mode, s);
  }
  if (m.nb <= 1024) return launch_mv<KIND, 1, 2>(m, T, x, ldx, y, ldy, mode, s);
  set_error("matvec: %d columns exceed the supported 32768", m.cols);
  return TN_EUNSUPPORTED;
}

int matvec(const Matrix& m, int T, const float* x, int ldx, float* y, int ldy, int mode, int* err,
           void* gemm_scratch, size_t gemm_scratch_bytes, cudaStream_t s) {
  if (T <= 0) return TN_OK;
  if (mode == EPI_SWIGLU) TN_REQUIRE((m.rows & 1) == 0, TN_EINVAL, "swiglu needs paired rows");
  switch (m.kind) {
    case MK_Q4:
    case MK_Q8:
      if (gemm_ok(m, T) && gemm_scratch)
        return gemm(m, T, x, ldx, nullptr, y, ldy, mode, gemm_scratch, gemm_scratch_bytes, err, s);
      return matvec_dec(m, T, x, ldx, y, ldy, mode, MvFuse(), err, s);
    case MK_F16: return matvec_kind<MK_F16>(m, T, x, ldx, y, ldy, mode, s);
    default: return matvec_kind<MK_F32>(m, T, x, ldx, y, ldy, mode, s);
  }
}

// ================================================================ rmsnorm
// web/inference-worker.js:516-522, sum of squares and the scale in double.
__global__ void k_rmsnorm(const float* __restrict__ h, int ldh, const int* __restrict__ rowsel,
                          const float* __restrict__ w, float* __restrict__ out, int ldo, int H) {
  const int t = blockIdx.x;
  const float* x = h + (size_t)(rowsel ? rowsel[t] : t) * ldh;
  double ss = 0.0;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const double v = x[i];
    ss += v * v;
  }
  __shared__ double part[32];
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    double v = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.0;
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) part[0] = v;
  }
  __syncthreads();
  const double inv = 1.0 / sqrt(part[0] / H + 1e-5);
  float* o = out + (size_t)t * ldo;
  for (int i = threadIdx.x; i < H; i += blockDim.x)
    o[i] = (float)__dmul_rn(__dmul_rn((double)x[i], inv), (double)w[i]);
}

int rmsnorm(const float* h, int ldh, const int* rowsel, const float* w, float* out, int ldo, int H,
            int T, cudaStream_t s) {
  if (T <= 0) return TN_OK;
  const int threads = H >= 4096 ? 1024 : (H >= 1024 ? 512 : 256);
  k_rmsnorm<<<T, threads, 0, s>>>(h, ldh, rowsel, w, out, ldo, H);
  TN_CHECK_LAUNCH();
  return TN_OK;
}

// ================================================================ embed
// embedLookup (web/inference-worker.js:509-515) from the repacked embed table
// grid (row, column block): one element per thread
__global__ void k_embed(int kind, const uint8_t* data, int vocab, int H, int nb, int cols_pad,
                        const int* __restrict__ ids, float* __restrict__ out, int ldo, int* err) {
  const int t = blockIdx.x, c = blockIdx.y * blockDim.x + threadIdx.x;
  const int id = ids[t];
  const bool ok = id >= 0 && id < vocab;
  if (!ok && c == 0) atomicExch(err, 1);
  if (c < H) out[(size_t)t * ldo + c] = ok ? mat_elem(kind, data, nb, cols_pad, (uint64_t)id, c) : 0.f;
}

int embed_rows(const Matrix& emb, const int* ids, int T, float* out, int ldo, int* d_err,
               cudaStream_t s) {
  if (T <= 0) return TN_OK;
  k_embed<<<dim3(T, (emb.cols + 255) / 256), 256, 0, s>>>(emb.kind, emb.data, emb.rows, emb.cols, emb.nb,
                                                          emb.cols_pad, ids, out, ldo, d_err);
  TN_CHECK_LAUNCH();
  return TN_OK;
}

// ================================================================ RoPE + KV append
// cos/sin of pos * theta^(-2i/hd) in double, once per step (web/inference-worker.js:533-534)
__global__ void k_rope_table(const RowInfo* __restrict__ rows, const double* __restrict__ freq, int half,
                             int T, double2* __restrict__ cs) {
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= T * half) return;
  const int t = k / half, i = k % half;
  const double ang = __dmul_rn((double)rows[t].pos, freq[i]);
  double sn, cn;
  sincos(ang, &sn, &cn);
  cs[k] = make_double2(cn, sn);
}

int rope_table(const RowInfo* rows, const double* freq, int half, int T, double2* cs, cudaStream_t s) {
  if (T <= 0) return TN_OK;
  k_rope_table<<<(T * half + 255) / 256, 256, 0, s>>>(rows, freq, half, T, cs);
  TN_CHECK_LAUNCH();
  return TN_OK;
}

// ropeCpu (web/inference-worker.js:528-540) on q and k, then the KV push of
// :554 into the cache at the row's KV index.  Rotations in double, unfused.
__global__ void k_rope_kv(const float* __restrict__ qkv, int ldqkv, const RowInfo* __restrict__ rows,
                          const double2* __restrict__ cs, float* __restrict__ q_out, void* __restrict__ kc,
                          void* __restrict__ vc, int kv_type, const KvMap kv, int nH, int nKV, int hd) {
  const int t = blockIdx.x;
  const RowInfo ri = rows[t];
  const int half = hd >> 1, qDim = nH * hd, kvDim = nKV * hd;
  const float* src = qkv + (size_t)t * ldqkv;
  const double2* c = cs + (size_t)t * half;
  const int nq = nH * half, nk = nKV * half;
  for (int k = threadIdx.x; k < nq + nk + kvDim; k += blockDim.x) {
    if (k < nq + nk) {
      const bool isq = k < nq;
      const int kk = isq ? k : k - nq;
      const int head = kk / half, i = kk % half;
      // q and k rows are stored pair-interleaved (dst_row): pair i at 2i, 2i + 1
      const float* base = src + (isq ? 0 : qDim) + head * hd;
      const double a = base[2 * i], b = base[2 * i + 1];
      const double2 r = c[i];
      const float o0 = (float)__dsub_rn(__dmul_rn(a, r.x), __dmul_rn(b, r.y));
      const float o1 = (float)__dadd_rn(__dmul_rn(a, r.y), __dmul_rn(b, r.x));
      if (isq) {
        float* qo = q_out + (size_t)t * qDim + head * hd;
        qo[i] = o0;
        qo[half + i] = o1;
      } else {
        const size_t ko = kv_row_off(kv, ri.slot, head, ri.kv_idx, hd);
        kv_store(kc, ko + i, kv_type, o0);
        kv_store(kc, ko + half + i, kv_type, o1);
      }
    } else {
      const int d = k - nq - nk, head = d / hd, e = d % hd;
      kv_store(vc, kv_row_off(kv, ri.slot, head, ri.kv_idx, hd) + e, kv_type, src[qDim + kvDim + d]);
    }
  }
}

int rope_kv(const float* qkv, int ldqkv, const RowInfo* rows, const double2* cs, float* q_out, void* kc, void* vc,
            int kv_type, const KvMap& kv, int nH, int nKV, int hd, int T, cudaStream_t s) {
  if (T <= 0) return TN_OK;
  k_rope_kv<<<T, 256, 0, s>>>(qkv, ldqkv, rows, cs, q_out, kc, vc, kv_type, kv, nH, nKV, hd);
  TN_CHECK_LAUNCH();
  return TN_OK;
}

// ================================================================ hop codec
__global__ void k_hop_encode(const float* __restrict__ h, int ldh, const int* __restrict__ rowsel, int H,
                             uint16_t* __restrict__ out) {
  const int t = blockIdx.y;
  const float* src = h + (size_t)(rowsel ? rowsel[t] : t) * ldh;
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < H; c += gridDim.x * blockDim.x)
    out[(size_t)t * H + c] = hop_encode(src[c]);
}

int hop_encode_rows(const float* h, int ldh, const int* rowsel, int T, int H, uint16_t* out,
                    cudaStream_t s) {
  if (T <= 0) return TN_OK;
  k_hop_encode<<<dim3((H + 255) / 256, T), 256, 0, s>>>(h, ldh, rowsel, H, out);
  TN_CHECK_LAUNCH();
  return TN_OK;
}

__global__ void k_hop_encode_flat(const float* __restrict__ in, uint64_t n, uint16_t* __restrict__ out) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    out[i] = hop_encode(in[i]);
}

int hop_encode_flat(const float* in, uint64_t n, uint16_t* out, cudaStream_t s) {
  if (n == 0) return TN_OK;
  const unsigned grid = (unsigned)std::min<uint64_t>((n + 255) / 256, 148ull * 64);
  k_hop_encode_flat<<<grid, 256, 0, s>>>(in, n, out);
  TN_CHECK_LAUNCH();
  return TN_OK;
}

__global__ void k_hop_decode(const uint16_t* __restrict__ in, uint64_t n, float* __restrict__ out) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    out[i] = f16_to_f32(in[i]);
}

int hop_decode(const uint16_t* in, uint64_t n, float* out, cudaStream_t s) {
  if (n == 0) return TN_OK;
  const unsigned grid = (unsigned)std::min<uint64_t>((n + 255) / 256, 148ull * 32);
  k_hop_decode<<<grid, 256, 0, s>>>(in, n, out);
  TN_CHECK_LAUNCH();
  return TN_OK;
}

// ================================================================ sampling
// web/inference-worker.js:658-672.  One CTA per row.  Greedy: lowest index
// among the maxima (NaN never compares greater).  Temperature: probabilities
// as the reference forms them (double exp, float store, double sum), then the
// nucleus and the draw located by bisection on the float bit patterns of the
// probabilities instead of a full sort; ties keep index order, as V8's stable
// sort does.
constexpr int SAMPLE_THREADS = 1024;

__device__ __forceinline__ double block_sum_d(double v, double* sh) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    double w = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.0;
    for (int o = 16; o > 0; o >>= 1) w += __shfl_xor_sync(0xffffffffu, w, o);
    if (threadIdx.x == 0) sh[32] = w;
  }
  __syncthreads();
  return sh[32];
}

__device__ __forceinline__ void argmax_merge(float& bv, int& bi, float v, int i) {
  if (v > bv || (v == bv && i < bi)) {
    bv = v;
    bi = i;
  }
}

// sum of p over elements with (bits(p) >= lo_bits) [and, if hi_excl, bits(p) < hi_bits]
__device__ double mass_ge(const float* p, int n, uint32_t lo_bits, double* sh) {
  double s = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = p[i];
    if (__float_as_uint(v) >= lo_bits) s += (double)v;
  }
  return block_sum_d(s, sh);
}

// first element (index order) among those with value bits == vb whose running
// sum, started at `start`, reaches `target`; -1 if none.
__device__ int tie_walk(const float* p, int n, uint32_t vb, double start, double target, double* total) {
  // single thread walk: ties are rare (exactly equal probabilities)
  double acc = start;
  int found = -1;
  for (int i = 0; i < n; i++) {
    if (__float_as_uint(p[i]) != vb) continue;
    acc += (double)p[i];
    if (found < 0 && acc >= target) found = i;
  }
  *total = acc;
  return found;
}

__global__ void __launch_bounds__(SAMPLE_THREADS) k_sample(float* __restrict__ logits, int vocab,
                                                           const double* __restrict__ params,
                                                           int* __restrict__ out) {
  __shared__ double shd[33];
  __shared__ float shv[32];
  __shared__ int shi[32];
  __shared__ int sh_int[2];
  const int row = blockIdx.x;
  float* l = logits + (size_t)row * vocab;
  const double temperature = params[3 * row], top_p = params[3 * row + 1], u = params[3 * row + 2];
  const int tid = threadIdx.x;

  // max (and argmax for greedy): four independent running maxima per thread
  // over 16-byte loads, so the loads of a thread are in flight together
  float bv = -INFINITY;
  int bi = 0;
  if ((vocab & 3) == 0) {
    const float4* l4 = reinterpret_cast<const float4*>(l);
    const int n4 = vocab >> 2;
    float v4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
    int i4[4] = {0, 0, 0, 0};
    for (int j = tid; j < n4; j += blockDim.x) {
      const float4 q = l4[j];
      argmax_merge(v4[0], i4[0], q.x, 4 * j);
      argmax_merge(v4[1], i4[1], q.y, 4 * j + 1);
      argmax_merge(v4[2], i4[2], q.z, 4 * j + 2);
      argmax_merge(v4[3], i4[3], q.w, 4 * j + 3);
    }
#pragma unroll
    for (int k = 0; k < 4; k++) argmax_merge(bv, bi, v4[k], i4[k]);
  } else {
    for (int i = tid; i < vocab; i += blockDim.x) argmax_merge(bv, bi, l[i], i);
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    argmax_merge(bv, bi, ov, oi);
  }
  if ((tid & 31) == 0) {
    shv[tid >> 5] = bv;
    shi[tid >> 5] = bi;
  }
  __syncthreads();
  if (tid < 32) {
    bv = tid < (blockDim.x >> 5) ? shv[tid] : -INFINITY;
    bi = tid < (blockDim.x >> 5) ? shi[tid] : 0;
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      argmax_merge(bv, bi, ov, oi);
    }
    if (tid == 0) {
      shv[0] = bv;
      shi[0] = bi;
    }
  }
  __syncthreads();
  if (!(temperature > 0.0)) {
    if (tid == 0) out[row] = shi[0];
    return;
  }
  const double mx = (double)shv[0];
  // probs: e = exp((l - mx) / T) (double), stored float; sum of the double e
  double s = 0.0;
  for (int i = tid; i < vocab; i += blockDim.x) {
    const double e = exp(((double)l[i] - mx) / temperature);
    l[i] = (float)e;
    s += e;
  }
  const double sum = block_sum_d(s, shd);
  for (int i = tid; i < vocab; i += blockDim.x) l[i] = (float)((double)l[i] / sum);
  __syncthreads();

  // nucleus: v* = largest value with mass(p >= v*) >= top_p
  const double total = mass_ge(l, vocab, 0u, shd);
  uint32_t vstar;
  double cum;  // reference's `cum` at the cut
  if (total < top_p) {
    vstar = 0u;  // every element is kept
    cum = total;
  } else {
    uint32_t lo = 0u, hi = 0x3f800001u;  // mass(lo) >= top_p > mass(hi)
    while (hi - lo > 1u) {
      const uint32_t mid = lo + (hi - lo) / 2u;
      if (mass_ge(l, vocab, mid, shd) >= top_p) lo = mid;
      else hi = mid;
    }
    vstar = lo;
    const double gt = mass_ge(l, vocab, vstar + 1u, shd);
    if (tid == 0) {
      double tot;
      const int cut_i = tie_walk(l, vocab, vstar, gt, top_p, &tot);
      // cum through the cut element: ties walked up to cut_i
      double acc = gt;
      for (int i = 0; i < vocab && cut_i >= 0; i++) {
        if (__float_as_uint(l[i]) != vstar) continue;
        acc += (double)l[i];
        if (i == cut_i) break;
      }
      shd[0] = cut_i >= 0 ? acc : tot;
      sh_int[0] = cut_i;
    }
    __syncthreads();
    cum = shd[0];
    __syncthreads();
  }
  // draw: r = u * cum; first element in sorted order whose running sum >= r
  const double r = u * cum;
  const double gt_star = mass_ge(l, vocab, vstar + 1u, shd);
  int pick = -1;
  if (gt_star >= r && vstar != 0x7fffffffu) {
    // among elements > v*: w = largest value with mass(p >= w) >= r
    uint32_t lo = vstar + 1u, hi = 0x3f800001u;
    if (mass_ge(l, vocab, lo, shd) >= r) {
      while (hi - lo > 1u) {
        const uint32_t mid = lo + (hi - lo) / 2u;
        if (mass_ge(l, vocab, mid, shd) >= r) lo = mid;
        else hi = mid;
      }
      const double before = mass_ge(l, vocab, lo + 1u, shd);
      if (tid == 0) {
        double tot;
        sh_int[1] = tie_walk(l, vocab, lo, before, r, &tot);
      }
      __syncthreads();
      pick = sh_int[1];
    }
  }
  if (pick < 0) {
    if (tid == 0) {
      double tot;
      const int k = tie_walk(l, vocab, vstar, gt_star, r, &tot);
      sh_int[1] = k;
    }
    __syncthreads();
    pick = sh_int[1];
  }
  if (tid == 0) out[row] = pick >= 0 ? pick : shi[0];
}

int sample_rows(float* logits, int n_rows, int vocab, const double* d_params, int* out, cudaStream_t s) {
  if (n_rows <= 0) return TN_OK;
  k_sample<<<n_rows, SAMPLE_THREADS, 0, s>>>(logits, vocab, d_params, out);
  TN_CHECK_LAUNCH();
  return TN_OK;
}

}  // namespace tn
