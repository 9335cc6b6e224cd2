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

// block-aligned q4_0 / q8_0 source: one thread per (row, block)
__global__ void k_repack_q(const uint8_t* __restrict__ src, int quant, int src_rows, int nb,
                           int dst_off, int dst_stride, uint8_t* __restrict__ data,
                           uint16_t* __restrict__ scales) {
  const uint64_t total = (uint64_t)src_rows * nb;
  const int bb = quant == TN_QUANT_Q8_0 ? 34 : 18, qb = bb - 2;
  for (uint64_t k = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; k < total;
       k += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t r = k / nb, b = k % nb;
    const uint8_t* blk = src + k * bb;
    const uint64_t dr = dst_row(r, dst_off, dst_stride);
    uint8_t* dq = data + (dr * nb + b) * qb;
    for (int j = 0; j < qb; j++) dq[j] = blk[2 + j];
    scales[dr * nb + b] = (uint16_t)(blk[0] | (blk[1] << 8));
  }
}

// same, for a 2-byte aligned source (every block then starts on an even
// address): 16-bit loads, one or two 16-byte stores per block
template <int QB>
__global__ void k_repack_q16(const uint16_t* __restrict__ src, int src_rows, int nb, int dst_off,
                             int dst_stride, uint4* __restrict__ data, uint16_t* __restrict__ scales) {
  constexpr int BW = QB / 2 + 1;  // 16-bit words per block
  const uint64_t total = (uint64_t)src_rows * nb;
  for (uint64_t k = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; k < total;
       k += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t r = k / nb, b = k % nb;
    const uint16_t* blk = src + k * BW;
    const uint64_t dr = dst_row(r, dst_off, dst_stride);
    uint32_t w[QB / 4];
#pragma unroll
    for (int j = 0; j < QB / 4; j++) w[j] = (uint32_t)blk[1 + 2 * j] | ((uint32_t)blk[2 + 2 * j] << 16);
    uint4* dq = data + (dr * nb + b) * (QB / 16);
#pragma unroll
    for (int v = 0; v < QB / 16; v++) dq[v] = make_uint4(w[4 * v], w[4 * v + 1], w[4 * v + 2], w[4 * v + 3]);
    scales[dr * nb + b] = blk[0];
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
static void mvd_prepare(Matrix* m);

int matrix_alloc(Matrix* m, int src_quant, int rows, int cols, cudaStream_t s) {
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
  const size_t dbytes = (size_t)m->rows_pad * m->nb * kind_block_bytes(m->kind);
  const size_t sbytes = (m->kind == MK_Q4 || m->kind == MK_Q8) ? (size_t)m->rows_pad * m->nb * 2 : 0;
  TN_CHECK_CUDA(cudaMalloc(&m->data, dbytes));
  // zero padding rows/columns on the stream the repack kernels will use
  TN_CHECK_CUDA(cudaMemsetAsync(m->data, 0, dbytes, s));
  if (sbytes) {
    TN_CHECK_CUDA(cudaMalloc(&m->scales, sbytes));
    TN_CHECK_CUDA(cudaMemsetAsync(m->scales, 0, sbytes, s));
  }
  m->bytes = dbytes + sbytes;
  num_sms();
  mv_prepare(m);
  mvd_prepare(m);
  return TN_OK;
}

int matrix_repack(Matrix* m, const uint8_t* d_src, int src_quant, int src_rows, int dst_off,
                  int dst_stride, cudaStream_t s) {
  TN_REQUIRE(dst_stride != 0 && (dst_stride > 0 || src_rows % (-dst_stride) == 0), TN_EINVAL,
             "matrix_repack: bad row stride %d", dst_stride);
  TN_REQUIRE(dst_off + (int64_t)(src_rows - 1) * (dst_stride > 0 ? dst_stride : 1) < m->rows, TN_EINVAL,
             "matrix_repack: rows out of range");
  const int grid = std::min(148 * 32, (int)std::max<int64_t>(1, ((int64_t)src_rows * m->nb + 255) / 256));
  const bool even = (reinterpret_cast<uintptr_t>(d_src) & 1) == 0;
  if (m->kind == MK_Q4 && even) {
    k_repack_q16<16><<<grid, 256, 0, s>>>((const uint16_t*)d_src, src_rows, m->nb, dst_off, dst_stride,
                                          (uint4*)m->data, m->scales);
  } else if (m->kind == MK_Q8 && even) {
    k_repack_q16<32><<<grid, 256, 0, s>>>((const uint16_t*)d_src, src_rows, m->nb, dst_off, dst_stride,
                                          (uint4*)m->data, m->scales);
  } else if (m->kind == MK_Q4 || m->kind == MK_Q8) {
    k_repack_q<<<grid, 256, 0, s>>>(d_src, src_quant, src_rows, m->nb, dst_off, dst_stride, m->data,
                                    m->scales);
  } else {
    k_repack_plain<<<grid, 256, 0, s>>>(d_src, src_quant, src_rows, m->cols, m->cols_pad, dst_off,
                                        dst_stride, m->kind, m->data);
  }
  TN_CHECK_LAUNCH();
  return TN_OK;
}

void matrix_free(Matrix* m) {
  if (m->data) cudaFree(m->data);
  if (m->scales) cudaFree(m->scales);
  m->data = nullptr;
  m->scales = nullptr;
  m->bytes = 0;
}

// value of element (r, c) of a repacked matrix
__device__ __forceinline__ float mat_elem(int kind, const uint8_t* data, const uint16_t* scales,
                                          int nb, int cols_pad, uint64_t r, int c) {
  if (kind == MK_F32) return ((const float*)data)[r * cols_pad + c];
  if (kind == MK_F16) return f16_to_f32(((const uint16_t*)data)[r * cols_pad + c]);
  const int b = c >> 5, j = c & 31;
  const float d = f16_to_f32(scales[r * nb + b]);
  if (kind == MK_Q8) return (float)(int8_t)data[(r * nb + b) * 32 + j] * d;
  const uint8_t byte = data[(r * nb + b) * 16 + (j >> 1)];
  return (float)(((j & 1) ? (byte >> 4) : (byte & 15)) - 8) * d;
}

__global__ void k_dequant(int kind, const uint8_t* data, const uint16_t* scales, int rows, int cols,
                          int nb, int cols_pad, float* out) {
  const uint64_t total = (uint64_t)rows * cols;
  for (uint64_t k = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; k < total;
       k += (uint64_t)gridDim.x * blockDim.x)
    out[k] = mat_elem(kind, data, scales, nb, cols_pad, k / cols, (int)(k % cols));
}

int matrix_dequant(const Matrix& m, float* out, cudaStream_t s) {
  const int grid = std::min(148 * 32, (int)std::max<int64_t>(1, ((int64_t)m.rows * m.cols + 255) / 256));
  k_dequant<<<grid, 256, 0, s>>>(m.kind, m.data, m.scales, m.rows, m.cols, m.nb, m.cols_pad, out);
  TN_CHECK_LAUNCH();
  return TN_OK;
}

// ================================================================ matvec
// CUDA-core dequant-matvec for few tokens (decode).  Each thread of a CTA
// owns NBT 32-wide block columns of K and keeps x for them in registers; the
// CTA walks a contiguous range of 8-row groups, streaming weights with 128-bit
// loads (rows are contiguous in K, so a warp's loads are 512 contiguous bytes),
// and reduces each group's 8 x TT partial dot products with a warp
// reduce-scatter plus one shared-memory pass.
//
// q4_0 decode without integer->float conversions: a nibble n placed in bits
// 16..19 of the float 0x3F000000 is 0.5 + n/256 (one PRMT), so per block
//   sum_j (n_j - 8) x_j = 256 * sum_j f_j x_j - 136 * sum_j x_j
// and sum_j x_j is computed once per x tile.
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

__device__ __forceinline__ float q4_f(uint32_t bytes4, int m) {
  // byte m of bytes4 (a nibble value) into bits 16..23 of 0x3F000000
  return __uint_as_float(__byte_perm(bytes4, 0x3F000000u, 0x7044u | ((uint32_t)m << 8)));
}
__device__ __forceinline__ float q8_f(uint32_t biased4, int m) {
  // byte m of (q ^ 0x80) as the low byte of 0x4B000000 -> 2^23 + q + 128
  return __uint_as_float(__byte_perm(biased4, 0x4B000000u, 0x7440u | (uint32_t)m));
}

template <int KIND, int TT, int NBT>
__global__ void __launch_bounds__(512) k_matvec(const uint8_t* __restrict__ data,
                                                const uint16_t* __restrict__ scales, int rows,
                                                int rows_pad, int cols, int nb, int T,
                                                const float* __restrict__ x, int ldx,
                                                float* __restrict__ y, int ldy, int mode) {
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
    float xs[TT][NBT];
#pragma unroll
    for (int tt = 0; tt < TT; tt++)
#pragma unroll
      for (int j = 0; j < NBT; j++) {
        const int b = tid + j * blockDim.x;
        const bool ok = b < nb && t0 + tt < T;
        float s = 0.f;
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
          s += (v.x + v.y) + (v.z + v.w);
        }
        xs[tt][j] = (KIND == MK_Q4) ? -136.f * s : s;
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
            float d[RG];
            if (KIND == MK_Q4 || KIND == MK_Q8) {
#pragma unroll
              for (int i = 0; i < RG; i++)
                d[i] = __half2float(__ushort_as_half(scales[(size_t)(g * 8 + rs + i) * nb + b]));
            }
#pragma unroll
            for (int i = 0; i < RG; i++) {
#pragma unroll
              for (int tt = 0; tt < TT; tt++) {
                float s = 0.f;
                if (KIND == MK_Q4) {
#pragma unroll
                  for (int k = 0; k < 4; k++) {
                    const uint32_t lo = w[i][k] & 0x0F0F0F0Fu, hi = (w[i][k] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
                    for (int m = 0; m < 4; m++) {
                      s = fmaf(q4_f(lo, m), xr[tt][j][8 * k + 2 * m], s);
                      s = fmaf(q4_f(hi, m), xr[tt][j][8 * k + 2 * m + 1], s);
                    }
                  }
                  acc[rs + i][tt] = fmaf(d[i], fmaf(256.f, s, xs[tt][j]), acc[rs + i][tt]);
                } else if (KIND == MK_Q8) {
#pragma unroll
                  for (int k = 0; k < 8; k++) {
                    const uint32_t bq = w[i][k] ^ 0x80808080u;
#pragma unroll
                    for (int m = 0; m < 4; m++)
                      s = fmaf(q8_f(bq, m) - 8388736.0f, xr[tt][j][4 * k + m], s);
                  }
                  acc[rs + i][tt] = fmaf(d[i], s, acc[rs + i][tt]);
                } else if (KIND == MK_F16) {
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
  k_matvec<KIND, TT, NBT><<<grid, mv_threads<KIND, TT, NBT>(m), 0, s>>>(m.data, m.scales, m.rows, m.rows_pad,
                                                                          m.cols, m.nb, T, x, ldx, y, ldy, mode);
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
  switch (m->kind) {
    case MK_Q4: mv_prepare_kind<MK_Q4>(m); break;
    case MK_Q8: mv_prepare_kind<MK_Q8>(m); break;
    case MK_F16: mv_prepare_kind<MK_F16>(m); break;
    default: mv_prepare_kind<MK_F32>(m); break;
  }
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

int matvec(const Matrix& m, int T, const float* x, int ldx, float* y, int ldy, int mode,
           cudaStream_t s) {
  if (T <= 0) return TN_OK;
  if (mode == EPI_SWIGLU) TN_REQUIRE((m.rows & 1) == 0, TN_EINVAL, "swiglu needs paired rows");
  switch (m.kind) {
    case MK_Q4: return matvec_kind<MK_Q4>(m, T, x, ldx, y, ldy, mode, s);
    case MK_Q8: return matvec_kind<MK_Q8>(m, T, x, ldx, y, ldy, mode, s);
    case MK_F16: return matvec_kind<MK_F16>(m, T, x, ldx, y, ldy, mode, s);
    default: return matvec_kind<MK_F32>(m, T, x, ldx, y, ldy, mode, s);
  }
}

// ================================================================ decode matvec
// Programmatic dependent launch: a kernel lets its successor start as soon as
// every CTA of it is running, and the successor streams weights (which no
// kernel writes) before it waits for its predecessor's results.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// ---- mbarrier + bulk-copy (TMA) primitives
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: gives up after ~2 s (or when another thread of the CTA gave
// up), raising the CTA's abort flag; callers then stop and report an error.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  const long long t0 = clock64();
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 255u) {
      if (*abort_flag) return false;
      if (clock64() - t0 > 4000000000ll) {
        *abort_flag = 1;
        return false;
      }
    }
  }
}
// global -> shared bulk copy completing on an mbarrier (16-byte aligned, size % 16 == 0)
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void consumer_sync(int nthreads) {
  asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}

struct MvdArgs {
  const uint8_t* data;
  const uint16_t* scales;
  int rows, rows_pad, cols, nb, T;
  const float* x;
  int ldx;
  float* y;
  int ldy, mode;
  int stages;       // shared-memory ring depth
  uint32_t stage_bytes;
  int* err;         // set to 1 if a bounded wait gave up
  MvFuse f;
};

// epilogue of rows [row0, row0 + nrows), whose per-warp partials are in red
template <int TT>
__device__ __forceinline__ void mvd_epilogue(const MvdArgs& a, const float* red, int red_stride, int nw, int row0,
                                             int nrows, int tid, int NT) {
  for (int e = tid; e < nrows * TT; e += NT) {
    const int r = e / TT, tt = e % TT, row = row0 + r;
    if (row >= a.rows || tt >= a.T) continue;
    const bool paired = (a.mode == EPI_SWIGLU || (a.mode == EPI_QKV_ROPE && row < a.f.q_dim + a.f.kv_dim));
    if (paired && (row & 1)) continue;  // handled with its even partner
    float s = 0.f, s2 = 0.f;
    for (int w2 = 0; w2 < nw; w2++) {
      s += red[w2 * red_stride + e];
      if (paired) s2 += red[w2 * red_stride + e + TT];
    }
    if (a.mode == EPI_STORE || a.mode == EPI_RESID) {
      float* py = a.y + (size_t)tt * a.ldy + row;
      *py = a.mode == EPI_RESID ? *py + s : s;
    } else if (a.mode == EPI_SWIGLU) {
      a.y[(size_t)tt * a.ldy + (row >> 1)] = (s / (1.0f + expf(-s))) * s2;
    } else {  // EPI_QKV_ROPE (web/inference-worker.js:528-540 and the KV push of :554)
      const MvFuse& f = a.f;
      const RowInfo ri = f.rinfo[tt];
      if (row < f.q_dim + f.kv_dim) {
        const bool isq = row < f.q_dim;
        const int rr = isq ? row : row - f.q_dim, head = rr / f.hd, i = (rr % f.hd) >> 1, half = f.hd >> 1;
        const double2 c = f.cs[(size_t)tt * half + i];
        const double av = s, bv = s2;
        const float o0 = (float)__dsub_rn(__dmul_rn(av, c.x), __dmul_rn(bv, c.y));
        const float o1 = (float)__dadd_rn(__dmul_rn(av, c.y), __dmul_rn(bv, c.x));
        float* dst = isq ? f.q_out + (size_t)tt * f.q_dim + head * f.hd
                         : f.kc + ri.slot * f.slot_stride + head * f.kvh_stride + (size_t)ri.kv_idx * f.hd;
        dst[i] = o0;
        dst[half + i] = o1;
      } else {
        const int dv = row - f.q_dim - f.kv_dim;
        f.vc[ri.slot * f.slot_stride + (dv / f.hd) * f.kvh_stride + (size_t)ri.kv_idx * f.hd + dv % f.hd] = s;
      }
    }
  }
}

// CUDA-core dequant-matvec for decode (1-2 tokens), fed by TMA bulk copies.
// A CTA owns a contiguous run of R-row units.  Thread 0 streams each unit's
// weights and scales (two contiguous bulk copies) into a ring of shared-memory
// stages guarded by full/empty mbarriers, refilling a stage as soon as every
// warp has released it, so ~5 units per SM are always in flight.  All threads
// consume: each owns NBT 32-wide block columns,
// keep x for them in registers, decode q4_0 / q8_0 from shared memory and
// reduce-scatter every unit's partial sums across the warp; one consumer
// barrier per 64 rows precedes the cross-warp sum and the fused epilogue.
//
// q4_0 decode without integer->float conversions: a nibble n placed in bits
// 16..19 of the float 0x3F000000 is 0.5 + n/256 (one PRMT), so per block
//   sum_j (n_j - 8) x_j = 256 * sum_j f_j x_j - 136 * sum_j x_j
// and sum_j x_j is computed once.
// d0 += a0 * b0, d1 += a1 * b1 with one packed f32x2 FMA (sm_100)
__device__ __forceinline__ void ffma2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
  asm("{\n .reg .b64 ra, rb, rc;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n mov.b64 rc, {%0, %1};\n"
      " fma.rn.f32x2 rc, ra, rb, rc;\n mov.b64 {%0, %1}, rc;\n}"
      : "+f"(d0), "+f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

constexpr int kMvtMaxStages = 8;

template <int KIND, int TT, int NBT, int R>
__global__ void __launch_bounds__(256, NBT == 1 ? 2 : 1) k_mvt(const MvdArgs a) {
  constexpr int BB = kind_block_bytes(KIND), W = BB / 4;
  constexpr int NV = R * TT;                    // values reduced per unit
  constexpr int LOGNV = NV == 2 ? 1 : (NV == 4 ? 2 : (NV == 8 ? 3 : (NV == 16 ? 4 : 5)));
  constexpr int SH = 5 - LOGNV;
  constexpr int CHU = 64 / R;                   // units per 64-row reduction chunk
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float red[2][8][64 * TT];
  __shared__ double nsum[8][TT];
  __shared__ int released[kMvtMaxStages];       // warps done with each stage's current unit
  __shared__ int last_unit[kMvtMaxStages];      // unit last issued into each stage
  __shared__ volatile int abort_flag;
  const int NT = blockDim.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = NT >> 5;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)a.stages * a.stage_bytes);
  const int NU = a.rows_pad / R;
  const int u0 = (int)((int64_t)NU * blockIdx.x / gridDim.x);
  const int nu = (int)((int64_t)NU * (blockIdx.x + 1) / gridDim.x) - u0;
  const uint32_t wbytes = (uint32_t)R * a.nb * BB, sbytes = (uint32_t)R * a.nb * 2;

  if (tid == 0) {
    abort_flag = 0;
    for (int s = 0; s < a.stages; s++) {
      mbar_init(&full[s], 1);
      released[s] = 0;
      last_unit[s] = -1;
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  pdl_launch_dependents();

  // issue unit k into its stage
  auto produce = [&](int k) {
    const int st = k % a.stages;
    uint8_t* dst = smem + (size_t)st * a.stage_bytes;
    const size_t row0 = (size_t)(u0 + k) * R;
    last_unit[st] = k;
    mbar_expect_tx(&full[st], wbytes + sbytes);
    bulk_g2s(dst, a.data + row0 * a.nb * BB, wbytes, &full[st]);
    bulk_g2s(dst + wbytes, a.scales + row0 * a.nb, sbytes, &full[st]);
  };
  if (tid == 0) {
    // weights do not depend on the previous kernel: start streaming at once
    for (int k = 0; k < nu && k < a.stages; k++) produce(k);
  }

  // ---------------- consumers
  pdl_wait();  // x is produced by the predecessor kernel
  float xr[TT][NBT][32];
  float xs[TT][NBT];
  double ss[TT];
#pragma unroll
  for (int tt = 0; tt < TT; tt++) {
    ss[tt] = 0.0;
    const bool tok = tt < a.T;
    const float* xrow = a.x + (size_t)(a.f.rowsel && tok ? a.f.rowsel[tt] : tt) * a.ldx;
#pragma unroll
    for (int j = 0; j < NBT; j++) {
      const int b = tid + j * NT;
      const bool ok = tok && b < a.nb;
#pragma unroll
      for (int e = 0; e < 32; e += 4) {
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (ok) v = *reinterpret_cast<const float4*>(xrow + b * 32 + e);
        xr[tt][j][e] = v.x;
        xr[tt][j][e + 1] = v.y;
        xr[tt][j][e + 2] = v.z;
        xr[tt][j][e + 3] = v.w;
        ss[tt] += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
      }
    }
  }
  if (a.f.norm_w) {
    // RMSNorm (web/inference-worker.js:516-522): the consumers hold the whole row
#pragma unroll
    for (int tt = 0; tt < TT; tt++) {
      double v = ss[tt];
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) nsum[warp][tt] = v;
    }
    consumer_sync(NT);
#pragma unroll
    for (int tt = 0; tt < TT; tt++) {
      double tot = 0.0;
      for (int w2 = 0; w2 < nw; w2++) tot += nsum[w2][tt];
      const double inv = 1.0 / sqrt(tot / a.cols + 1e-5);
#pragma unroll
      for (int j = 0; j < NBT; j++) {
        const int b = tid + j * NT;
        if (b < a.nb) {
#pragma unroll
          for (int e = 0; e < 32; e++)
            xr[tt][j][e] = (float)__dmul_rn(__dmul_rn((double)xr[tt][j][e], inv), (double)a.f.norm_w[b * 32 + e]);
        }
      }
    }
  }
#pragma unroll
  for (int tt = 0; tt < TT; tt++)
#pragma unroll
    for (int j = 0; j < NBT; j++) {
      float s = 0.f;
#pragma unroll
      for (int e = 0; e < 32; e++) s += xr[tt][j][e];
      xs[tt][j] = KIND == MK_Q4 ? -136.f * s : s;
    }

  // Every thread runs every iteration and barrier even after an abort (then
  // it only skips the math), so no thread can be left waiting at bar.sync.
  int rb = 0;
  for (int k = 0; k < nu; k++) {
    const int st = k % a.stages;
    const bool ready = mbar_wait(&full[st], (k / a.stages) & 1, &abort_flag);
    const uint8_t* wsm = smem + (size_t)st * a.stage_bytes;
    const uint16_t* ssm = reinterpret_cast<const uint16_t*>(wsm + wbytes);
    float acc[R][TT];
#pragma unroll
    for (int i = 0; i < R; i++) {
#pragma unroll
      for (int tt = 0; tt < TT; tt++) acc[i][tt] = 0.f;
#pragma unroll
      for (int j = 0; j < NBT; j++) {
        const int b = tid + j * NT;
        if (ready && b < a.nb) {
          uint32_t w[W];
#pragma unroll
          for (int v = 0; v < W / 4; v++) {
            const uint4 q = *reinterpret_cast<const uint4*>(wsm + ((size_t)i * a.nb + b) * BB + 16 * v);
            w[4 * v] = q.x;
            w[4 * v + 1] = q.y;
            w[4 * v + 2] = q.z;
            w[4 * v + 3] = q.w;
          }
          const float di = __half2float(__ushort_as_half(ssm[i * a.nb + b]));
#pragma unroll
          for (int tt = 0; tt < TT; tt++) {
            // even / odd elements in the two halves of packed f32x2 FMAs
            float s0 = 0.f, s1 = 0.f;
            if constexpr (KIND == MK_Q4) {
#pragma unroll
              for (int kk = 0; kk < 4; kk++) {
                const uint32_t lo = w[kk] & 0x0F0F0F0Fu, hi = (w[kk] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
                for (int m = 0; m < 4; m++)
                  ffma2(s0, s1, q4_f(lo, m), q4_f(hi, m), xr[tt][j][8 * kk + 2 * m], xr[tt][j][8 * kk + 2 * m + 1]);
              }
              acc[i][tt] = fmaf(di, fmaf(256.f, s0 + s1, xs[tt][j]), acc[i][tt]);
            } else {
#pragma unroll
              for (int kk = 0; kk < 8; kk++) {
                const uint32_t bq = w[kk] ^ 0x80808080u;
                ffma2(s0, s1, q8_f(bq, 0) - 8388736.0f, q8_f(bq, 1) - 8388736.0f, xr[tt][j][4 * kk],
                      xr[tt][j][4 * kk + 1]);
                ffma2(s0, s1, q8_f(bq, 2) - 8388736.0f, q8_f(bq, 3) - 8388736.0f, xr[tt][j][4 * kk + 2],
                      xr[tt][j][4 * kk + 3]);
              }
              acc[i][tt] = fmaf(di, s0 + s1, acc[i][tt]);
            }
          }
        }
      }
    }
    // this warp has read the stage: the last warp to release it refills it
    // with the unit `stages` ahead (nobody waits for the slowest warp)
    __syncwarp();
    if (lane == 0) {
      __threadfence_block();
      if (atomicAdd(&released[st], 1) == nw - 1) {
        __threadfence_block();
        released[st] = 0;
        const int kn = k + a.stages;
        if (kn < nu && !abort_flag) {
          // order every warp's reads of the stage before the copy that overwrites it
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          produce(kn);
        }
      }
    }
    float v[NV];
#pragma unroll
    for (int i = 0; i < R; i++)
#pragma unroll
      for (int tt = 0; tt < TT; tt++) v[i * TT + tt] = acc[i][tt];
    const float r = warp_reduce_scatter<NV>(v, lane);
    const int cu = k % CHU;
    if ((lane & ((1 << SH) - 1)) == 0) red[rb][warp][cu * NV + (lane >> SH)] = r;
    if (cu == CHU - 1 || k == nu - 1) {
      consumer_sync(NT);
      if (!abort_flag)
        mvd_epilogue<TT>(a, &red[rb][0][0], 64 * TT, nw, (u0 + k - cu) * R, (cu + 1) * R, tid, NT);
      rb ^= 1;
    }
  }
  consumer_sync(NT);
  if (tid == 0 && abort_flag) {
    // no copy may still be landing when the CTA exits
    for (int s = 0; s < a.stages; s++) {
      const int j = last_unit[s];
      if (j < 0) continue;
      abort_flag = 0;
      if (!mbar_wait(&full[s], (j / a.stages) & 1, &abort_flag)) break;
    }
    atomicExch(a.err, 1);
  }
}

// ---- launch configuration of the decode matvec of one matrix
static int mvt_nbt(int nb) { return nb <= 256 ? 1 : (nb <= 512 ? 2 : 4); }
// One block column per thread: 2 CTAs per SM, ~24 KB stages in ~96 KB rings;
// wider rows (more x registers per thread): 1 CTA per SM, ~48 KB stages.
static int mvt_ctas_target(int nb) { return mvt_nbt(nb) == 1 ? 2 : 1; }
static int mvt_rows(const Matrix& m) {  // R: rows per unit
  const int bb = kind_block_bytes(m.kind) + 2;
  const size_t cap = mvt_ctas_target(m.nb) == 2 ? 24576 : 49152;
  int r = 16;
  while (r > 2 && (size_t)r * m.nb * bb > cap) r >>= 1;
  return r;
}

template <int KIND, int TT, int NBT, int R>
static int mvt_occ(int threads, int smem) {
  int o = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, k_mvt<KIND, TT, NBT, R>, threads, smem) != cudaSuccess)
    o = 1;
  return o < 1 ? 1 : o;
}

template <int KIND, int TT, int NBT, int R>
static void mvt_set_smem(int bytes) {
  cudaFuncSetAttribute(k_mvt<KIND, TT, NBT, R>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

// sets the dynamic shared memory limit; returns resident CTAs per SM
template <int KIND, int TT, int NBT>
static int mvt_set_smem_r(int R, int bytes, int threads) {
  switch (R) {
    case 2: mvt_set_smem<KIND, TT, NBT, 2>(bytes); return mvt_occ<KIND, TT, NBT, 2>(threads, bytes);
    case 4: mvt_set_smem<KIND, TT, NBT, 4>(bytes); return mvt_occ<KIND, TT, NBT, 4>(threads, bytes);
    case 8: mvt_set_smem<KIND, TT, NBT, 8>(bytes); return mvt_occ<KIND, TT, NBT, 8>(threads, bytes);
    default: mvt_set_smem<KIND, TT, NBT, 16>(bytes); return mvt_occ<KIND, TT, NBT, 16>(threads, bytes);
  }
}

static void mvd_prepare(Matrix* m) {
  if (!(m->kind == MK_Q4 || m->kind == MK_Q8) || m->nb > 1024) return;
  const int R = mvt_rows(*m), nbt = mvt_nbt(m->nb);
  // every unit's scale run must start on a 16-byte boundary and be a multiple
  // of 16 bytes for the bulk copy (the weight run always is): else no decode kernel
  if (((size_t)R * m->nb * 2) % 16 != 0) return;
  const uint32_t stage = (uint32_t)(((size_t)R * m->nb * (kind_block_bytes(m->kind) + 2) + 127) & ~(size_t)127);
  const size_t ring = mvt_ctas_target(m->nb) == 2 ? 96 * 1024 : 200 * 1024;
  const int stages = (int)std::max<size_t>(2, std::min<size_t>(kMvtMaxStages, ring / stage));
  m->mvt_rows = R;
  m->mvt_stages = stages;
  m->mvt_stage_bytes = stage;
  m->mvt_smem = (int)(stages * stage + stages * sizeof(uint64_t));
  const int NT = ((m->nb + nbt - 1) / nbt + 31) & ~31;
  // (set once, outside any stream capture)
  int o1 = 1, o2 = 1;
  if (m->kind == MK_Q4) {
    if (nbt == 1) { o1 = mvt_set_smem_r<MK_Q4, 1, 1>(R, m->mvt_smem, NT); o2 = mvt_set_smem_r<MK_Q4, 2, 1>(R, m->mvt_smem, NT); }
    else if (nbt == 2) { o1 = mvt_set_smem_r<MK_Q4, 1, 2>(R, m->mvt_smem, NT); o2 = mvt_set_smem_r<MK_Q4, 2, 2>(R, m->mvt_smem, NT); }
    else o1 = o2 = mvt_set_smem_r<MK_Q4, 1, 4>(R, m->mvt_smem, NT);
  } else {
    if (nbt == 1) { o1 = mvt_set_smem_r<MK_Q8, 1, 1>(R, m->mvt_smem, NT); o2 = mvt_set_smem_r<MK_Q8, 2, 1>(R, m->mvt_smem, NT); }
    else if (nbt == 2) { o1 = mvt_set_smem_r<MK_Q8, 1, 2>(R, m->mvt_smem, NT); o2 = mvt_set_smem_r<MK_Q8, 2, 2>(R, m->mvt_smem, NT); }
    else o1 = o2 = mvt_set_smem_r<MK_Q8, 1, 4>(R, m->mvt_smem, NT);
  }
  m->mvt_ctas[0] = o1;
  m->mvt_ctas[1] = o2;
}

template <int KIND, int TT, int NBT, int R>
static int launch_mvt(const Matrix& m, int T, const float* x, int ldx, float* y, int ldy, int mode,
                      const MvFuse& f, int* err, cudaStream_t s) {
  const int NT = ((m.nb + NBT - 1) / NBT + 31) & ~31;
  const int NU = m.rows_pad / R;
  const int grid = std::max(1, std::min(NU, m.mvt_ctas[TT - 1] * num_sms()));
  const MvdArgs a{m.data, m.scales, m.rows, m.rows_pad, m.cols, m.nb, T, x, ldx, y, ldy, mode,
                  m.mvt_stages, m.mvt_stage_bytes, err, f};
  TN_CHECK_CUDA(launch_pdl(k_mvt<KIND, TT, NBT, R>, dim3(grid), dim3(NT), (size_t)m.mvt_smem, s, a));
  return TN_OK;
}

template <int KIND, int TT, int NBT>
static int launch_mvt_r(const Matrix& m, int T, const float* x, int ldx, float* y, int ldy, int mode,
                        const MvFuse& f, int* err, cudaStream_t s) {
  switch (m.mvt_rows) {
    case 2: return launch_mvt<KIND, TT, NBT, 2>(m, T, x, ldx, y, ldy, mode, f, err, s);
    case 4: return launch_mvt<KIND, TT, NBT, 4>(m, T, x, ldx, y, ldy, mode, f, err, s);
    case 8: return launch_mvt<KIND, TT, NBT, 8>(m, T, x, ldx, y, ldy, mode, f, err, s);
    default: return launch_mvt<KIND, TT, NBT, 16>(m, T, x, ldx, y, ldy, mode, f, err, s);
  }
}

bool matvec_dec_ok(const Matrix& m, int T) {
  if (!(m.kind == MK_Q4 || m.kind == MK_Q8) || m.nb > 1024 || T < 1 || m.mvt_rows == 0) return false;
  return T <= (mvt_nbt(m.nb) <= 2 ? 2 : 1);
}

template <int KIND>
static int matvec_dec_kind(const Matrix& m, int T, const float* x, int ldx, float* y, int ldy, int mode,
                           const MvFuse& f, int* err, cudaStream_t s) {
  switch (mvt_nbt(m.nb)) {
    case 1: return T == 1 ? launch_mvt_r<KIND, 1, 1>(m, T, x, ldx, y, ldy, mode, f, err, s)
                          : launch_mvt_r<KIND, 2, 1>(m, T, x, ldx, y, ldy, mode, f, err, s);
    case 2: return T == 1 ? launch_mvt_r<KIND, 1, 2>(m, T, x, ldx, y, ldy, mode, f, err, s)
                          : launch_mvt_r<KIND, 2, 2>(m, T, x, ldx, y, ldy, mode, f, err, s);
    default: return launch_mvt_r<KIND, 1, 4>(m, T, x, ldx, y, ldy, mode, f, err, s);
  }
}

int matvec_dec(const Matrix& m, int T, const float* x, int ldx, float* y, int ldy, int mode, const MvFuse& f,
               int* err, cudaStream_t s) {
  TN_REQUIRE(matvec_dec_ok(m, T), TN_EUNSUPPORTED, "matvec_dec: %d tokens of kind %d, %d columns", T, m.kind,
             m.cols);
  TN_REQUIRE((ldx & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0, TN_EINVAL,
             "matvec_dec: x rows must be 16-byte aligned");
  TN_REQUIRE(mode != EPI_SWIGLU || (m.rows & 1) == 0, TN_EINVAL, "swiglu needs paired rows");
  TN_REQUIRE(err, TN_EINVAL, "matvec_dec: error flag required");
  if (m.kind == MK_Q4) return matvec_dec_kind<MK_Q4>(m, T, x, ldx, y, ldy, mode, f, err, s);
  return matvec_dec_kind<MK_Q8>(m, T, x, ldx, y, ldy, mode, f, err, s);
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
__global__ void k_embed(int kind, const uint8_t* data, const uint16_t* scales, int vocab, int H, int nb,
                        int cols_pad, const int* __restrict__ ids, float* __restrict__ out, int ldo,
                        int* err) {
  const int t = blockIdx.x;
  const int id = ids[t];
  const bool ok = id >= 0 && id < vocab;
  if (!ok && threadIdx.x == 0) atomicExch(err, 1);
  for (int c = threadIdx.x; c < H; c += blockDim.x)
    out[(size_t)t * ldo + c] = ok ? mat_elem(kind, data, scales, nb, cols_pad, (uint64_t)id, c) : 0.f;
}

int embed_rows(const Matrix& emb, const int* ids, int T, float* out, int ldo, int* d_err,
               cudaStream_t s) {
  if (T <= 0) return TN_OK;
  k_embed<<<T, 256, 0, s>>>(emb.kind, emb.data, emb.scales, emb.rows, emb.cols, emb.nb, emb.cols_pad,
                            ids, out, ldo, d_err);
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
                          const double2* __restrict__ cs, float* __restrict__ q_out,
                          float* __restrict__ kc, float* __restrict__ vc, size_t slot_stride,
                          size_t kvh_stride, int nH, int nKV, int hd) {
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
        float* ko = kc + ri.slot * slot_stride + head * kvh_stride + (size_t)ri.kv_idx * hd;
        ko[i] = o0;
        ko[half + i] = o1;
      }
    } else {
      const int d = k - nq - nk, head = d / hd, e = d % hd;
      vc[ri.slot * slot_stride + head * kvh_stride + (size_t)ri.kv_idx * hd + e] =
          src[qDim + kvDim + d];
    }
  }
}

int rope_kv(const float* qkv, int ldqkv, const RowInfo* rows, const double2* cs, float* q_out, float* kc,
            float* vc, size_t slot_stride, size_t kvh_stride, int nH, int nKV, int hd, int T,
            cudaStream_t s) {
  if (T <= 0) return TN_OK;
  k_rope_kv<<<T, 256, 0, s>>>(qkv, ldqkv, rows, cs, q_out, kc, vc, slot_stride, kvh_stride, nH, nKV, hd);
  TN_CHECK_LAUNCH();
  return TN_OK;
}

// ================================================================ attention
// One-query GQA attention (web/inference-worker.js:556-564) as split-K
// flash-decoding: CTA (split, kv head, row) walks its slice of the row's
// cached positions in tiles of 32, serving all G query heads of the KV head
// from one copy of each K/V tile in shared memory; (max, sum, unnormalised
// output) partials are merged by k_attn_combine.
constexpr int ATT_TILE = 32;
constexpr int ATT_THREADS = 128;

template <int HD, int G>
__global__ void __launch_bounds__(ATT_THREADS)
    k_attn_split(const float* __restrict__ q, int ldq, const float* __restrict__ kc,
                 const float* __restrict__ vc, size_t slot_stride, size_t kvh_stride,
                 const RowInfo* __restrict__ rows, int nH, int n_splits, float scale,
                 float* __restrict__ part_o, float2* __restrict__ part_ml) {
  constexpr int HD4 = HD / 4;
  __shared__ __align__(16) float Ks[ATT_TILE][HD];
  __shared__ __align__(16) float Vs[ATT_TILE][HD];
  __shared__ __align__(16) float Qs[G][HD];
  __shared__ float Ps[G][ATT_TILE];
  __shared__ float alpha_s[G];
  const int split = blockIdx.x, kvh = blockIdx.y, t = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const RowInfo ri = rows[t];
  const int L = ri.len;
  const int lo = (int)((int64_t)L * split / n_splits), hi = (int)((int64_t)L * (split + 1) / n_splits);
  const float* kbase = kc + ri.slot * slot_stride + kvh * kvh_stride;
  const float* vbase = vc + ri.slot * slot_stride + kvh * kvh_stride;

  for (int k = tid; k < G * HD; k += ATT_THREADS)
    Qs[k / HD][k % HD] = q[(size_t)t * ldq + (kvh * G + k / HD) * HD + k % HD];

  // per-head running max / sum live in every lane of the warp owning the head
  float m_run[(G + 3) / 4], l_run[(G + 3) / 4];
#pragma unroll
  for (int i = 0; i < (G + 3) / 4; i++) {
    m_run[i] = -INFINITY;
    l_run[i] = 0.f;
  }
  constexpr int DPT = (G * HD + ATT_THREADS - 1) / ATT_THREADS;  // (head, dim) outputs per thread
  float acc[DPT];
#pragma unroll
  for (int i = 0; i < DPT; i++) acc[i] = 0.f;

  for (int p0 = lo; p0 < hi; p0 += ATT_TILE) {
    const int n = min(ATT_TILE, hi - p0);
    __syncthreads();
    for (int k = tid; k < ATT_TILE * HD4; k += ATT_THREADS) {
      const int p = k / HD4, j = k % HD4;
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
      if (p < n) {
        kv = *reinterpret_cast<const float4*>(kbase + (size_t)(p0 + p) * HD + 4 * j);
        vv = *reinterpret_cast<const float4*>(vbase + (size_t)(p0 + p) * HD + 4 * j);
      }
      *reinterpret_cast<float4*>(&Ks[p][4 * j]) = kv;
      *reinterpret_cast<float4*>(&Vs[p][4 * j]) = vv;
    }
    __syncthreads();
    // scores: thread (p = lane, heads warp, warp+4, ...)
    for (int g = warp; g < G; g += ATT_THREADS / 32) {
      float dot = 0.f;
      const int p = lane;
#pragma unroll 8
      for (int j0 = 0; j0 < HD4; j0++) {
        const int j = (j0 + p) % HD4;  // rotate to keep the 8 lanes of a phase on distinct banks
        const float4 kk = *reinterpret_cast<const float4*>(&Ks[p][4 * j]);
        const float4 qq = *reinterpret_cast<const float4*>(&Qs[g][4 * j]);
        dot = fmaf(qq.x, kk.x, dot);
        dot = fmaf(qq.y, kk.y, dot);
        dot = fmaf(qq.z, kk.z, dot);
        dot = fmaf(qq.w, kk.w, dot);
      }
      const float sc = p < n ? dot * scale : -INFINITY;
      float mx = sc;
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const int gi = g / (ATT_THREADS / 32);
      const float m_new = fmaxf(m_run[gi], mx);
      const float e = p < n ? expf(sc - m_new) : 0.f;
      float se = e;
      for (int o = 16; o > 0; o >>= 1) se += __shfl_xor_sync(0xffffffffu, se, o);
      const float al = expf(m_run[gi] - m_new);  // m_run = -inf on the first tile -> 0
      l_run[gi] = l_run[gi] * al + se;
      m_run[gi] = m_new;
      Ps[g][p] = e;
      if (lane == 0) alpha_s[g] = al;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < DPT; i++) {
      const int k = tid + i * ATT_THREADS;
      if (k < G * HD) {
        const int g = k / HD, d = k % HD;
        float a = acc[i] * alpha_s[g];
#pragma unroll 8
        for (int p = 0; p < ATT_TILE; p++) a = fmaf(Ps[g][p], Vs[p][d], a);
        acc[i] = a;
      }
    }
  }
  // partials: [(t * nH + head) * n_splits + split]
#pragma unroll
  for (int i = 0; i < DPT; i++) {
    const int k = tid + i * ATT_THREADS;
    if (k < G * HD) {
      const int g = k / HD, d = k % HD, head = kvh * G + g;
      part_o[(((size_t)t * nH + head) * n_splits + split) * HD + d] = acc[i];
    }
  }
  for (int g = warp; g < G; g += ATT_THREADS / 32) {
    const int gi = g / (ATT_THREADS / 32), head = kvh * G + g;
    if (lane == 0) part_ml[((size_t)t * nH + head) * n_splits + split] = make_float2(m_run[gi], l_run[gi]);
  }
}

__global__ void k_attn_combine(const float* __restrict__ part_o, const float2* __restrict__ part_ml,
                               int nH, int hd, int n_splits, float* __restrict__ out, int ldo) {
  const int head = blockIdx.x, t = blockIdx.y;
  const size_t base = ((size_t)t * nH + head) * n_splits;
  float M = -INFINITY;
  for (int s = 0; s < n_splits; s++) M = fmaxf(M, part_ml[base + s].x);
  float Lsum = 0.f;
  for (int s = 0; s < n_splits; s++) {
    const float2 ml = part_ml[base + s];
    if (ml.y > 0.f) Lsum += ml.y * expf(ml.x - M);
  }
  const float inv = Lsum > 0.f ? 1.0f / Lsum : 0.f;
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float o = 0.f;
    for (int s = 0; s < n_splits; s++) {
      const float2 ml = part_ml[base + s];
      if (ml.y > 0.f) o = fmaf(part_o[(base + s) * hd + d], expf(ml.x - M), o);
    }
    out[(size_t)t * ldo + head * hd + d] = o * inv;
  }
}

int attn_splits(int T, int nKV, int max_ctx) {
  const int want = (2 * num_sms() + T * nKV - 1) / (T * nKV);
  const int cap = std::max(1, (max_ctx + 127) / 128);
  return std::max(1, std::min(want, cap));
}

size_t attn_scratch_bytes(int T, int nH, int hd, int n_splits) {
  const size_t n = (size_t)T * nH * n_splits;
  return ((n * hd * sizeof(float) + 255) & ~(size_t)255) + n * sizeof(float2);
}

template <int HD>
static int launch_attn_hd(const float* q, int ldq, const float* kc, const float* vc, size_t slot_stride,
                          size_t kvh_stride, const RowInfo* rows, int T, int nH, int nKV, int G,
                          int n_splits, float* part_o, float2* part_ml, cudaStream_t s) {
  const dim3 grid(n_splits, nKV, T);
  const float scale = (float)(1.0 / sqrt((double)HD));
  switch (G) {
#define TN_ATT_CASE(g)                                                                             \
  case g:                                                                                          \
    k_attn_split<HD, g><<<grid, ATT_THREADS, 0, s>>>(q, ldq, kc, vc, slot_stride, kvh_stride, rows, nH, \
                                                     n_splits, scale, part_o, part_ml);            \
    break;
    TN_ATT_CASE(1)
    TN_ATT_CASE(2)
    TN_ATT_CASE(4)
    TN_ATT_CASE(8)
    TN_ATT_CASE(16)
#undef TN_ATT_CASE
    default:
      set_error("attention: %d query heads per KV head unsupported", G);
      return TN_EUNSUPPORTED;
  }
  TN_CHECK_LAUNCH();
  return TN_OK;
}

int attention(const float* q, int ldq, const float* kc, const float* vc, size_t slot_stride,
              size_t kvh_stride, const RowInfo* rows, int T, int nH, int nKV, int hd, int n_splits,
              float* out, int ldo, void* scratch, cudaStream_t s) {
  if (T <= 0) return TN_OK;
  TN_REQUIRE(nH % nKV == 0, TN_EUNSUPPORTED, "attention: n_heads %% n_kv_heads != 0");
  const int G = nH / nKV;
  const size_t n = (size_t)T * nH * n_splits;
  float* part_o = (float*)scratch;
  float2* part_ml = (float2*)((char*)scratch + ((n * hd * sizeof(float) + 255) & ~(size_t)255));
  int rc;
  switch (hd) {
    case 32: rc = launch_attn_hd<32>(q, ldq, kc, vc, slot_stride, kvh_stride, rows, T, nH, nKV, G, n_splits, part_o, part_ml, s); break;
    case 64: rc = launch_attn_hd<64>(q, ldq, kc, vc, slot_stride, kvh_stride, rows, T, nH, nKV, G, n_splits, part_o, part_ml, s); break;
    case 128: rc = launch_attn_hd<128>(q, ldq, kc, vc, slot_stride, kvh_stride, rows, T, nH, nKV, G, n_splits, part_o, part_ml, s); break;
    default: set_error("attention: head_dim %d unsupported", hd); return TN_EUNSUPPORTED;
  }
  if (rc) return rc;
  k_attn_combine<<<dim3(nH, T), std::min(hd, 128), 0, s>>>(part_o, part_ml, nH, hd, n_splits, out, ldo);
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

  // max (and argmax for greedy)
  float bv = -INFINITY;
  int bi = 0;
  for (int i = tid; i < vocab; i += blockDim.x) argmax_merge(bv, bi, l[i], i);
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
