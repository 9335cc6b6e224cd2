// tn_kernels.cuh -- device data structures and launchers of the stage engine.
#pragma once

#include <cuda.h>  // CUtensorMap (the encoder is fetched from the driver at run time)

#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "tn_common.cuh"

namespace tn {

// Device layouts of a [rows x cols] weight matrix after the init-time repack.
//   MK_Q4 / MK_Q8: tensor-core fragment order.  Rows are cut into tiles of 16
//           and the 32-element blocks of a row into pairs (2p, 2p + 1); every
//           (tile, pair) is one record of tile_a_bytes(kind) weight bytes plus
//           64 bytes of fp16 scales, tiles major, pairs minor.  Within a record,
//           lane l = 4 g + c (g = 0..7, c = 0..3) owns 16 (q4) / 32 (q8)
//           contiguous bytes: exactly the A operands of the two
//           mma.m16n8k32 (half h = 0, 1) that cover rows g and g + 8 of the
//           tile, A columns 0..15 being elements 16 h .. 16 h + 15 of block 2p
//           and columns 16..31 the same elements of block 2p + 1.
//             q4: word 2h + q, byte i = (s(row g) << 4) | s(row g + 8) for
//                 element 16 h + 4 c + i of block 2p + q, where s = nibble ^ 8
//                 is the weight's (n - 8) as a 4-bit two's complement value;
//             q8: word 4h + 2q + u, byte i = q8 value of row g + 8u, same element.
//           Scales: u32 (2 g + q) of the scale area = (row g, row g + 8) of block 2p + q.
//           Padding rows and blocks are zero, i.e. weight 0.
//   MK_F16: data [rows_pad][cols_pad]  fp16 bits (zero padded)
//   MK_F32: data [rows_pad][cols_pad]  f32 (zero padded); also holds exactly dequantised
//           q4_0/q8_0 tensors whose rows do not start on a block boundary
//   rows_pad is a multiple of 16.
enum MatKind { MK_Q4 = 0, MK_Q8 = 1, MK_F16 = 2, MK_F32 = 3 };

__host__ __device__ constexpr int tile_a_bytes(int k) { return k == MK_Q4 ? 512 : 1024; }
__host__ __device__ constexpr int tile_rec_bytes(int k) { return tile_a_bytes(k) + 64; }

// Programmatic dependent launch: a kernel lets its successor start as soon as
// every CTA of it is running, and the successor streams weights (which no
// kernel writes) before it waits for its predecessor's results.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
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
// launch_pdl with thread-block clusters of cluster_x CTAs along x
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, int cluster_x,
                                      cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = (unsigned)cluster_x;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// Launch shape of the tensor-core matvec for one token count (1, 2 or 4): K is
// cut into ks chunks of ckp block pairs (a chunk's activation digits fill one
// shared-memory table), a chunk into nsc sub-chunks of scp pairs (one
// shared-memory stage each).
struct MmShape {
  int ks = 0, ckp = 0, nsc = 0, scp = 0;
  int stages = 0, smem = 0, ctas = 1;  // ring depth, dynamic shared memory, resident CTAs per SM
  uint32_t stage_bytes = 0;
};

struct Matrix {
  int kind = MK_F32;
  int rows = 0, cols = 0;
  int rows_pad = 0, cols_pad = 0, nb = 0;
  int tiles = 0, pairs = 0;  // MK_Q4 / MK_Q8 record grid
  uint8_t* data = nullptr;
  size_t bytes = 0;
  int occ[2] = {0, 0};       // resident CTAs per SM of the CUDA-core matvec (MK_F16 / MK_F32)
  MmShape mm[3];             // tensor-core matvec (MK_Q4 / MK_Q8), 1, 2 and 4 token columns
  // cross-CTA partial sums [chunk][tile][part 0 / 1][32 x token pairs] and
  // per-tile arrival counters (zero between launches: the CTA that completes
  // a tile resets them).  Matrices whose launches are ordered on one stream
  // may share one pair of buffers (ws_owned false): every access follows the
  // wait for the previous kernel.
  size_t ws_floats = 0;
  float* ws = nullptr;
  size_t cnt_ints = 0;
  int* cnt = nullptr;
  bool ws_owned = true;
  // MK_Q4 / MK_Q8: TMA maps of the records as a [tiles][pairs][record] tensor,
  // boxes of 8 tiles x 1 / 2 / 4 pairs (wmap[0..2]: the GEMM's raw stages)
  CUtensorMap wmap[3];
  bool has_wmap = false;
};

// bytes per 32-element block of the data plane (row-major kinds)
__host__ __device__ constexpr int kind_block_bytes(int k) {
  return k == MK_Q4 ? 16 : (k == MK_Q8 ? 32 : (k == MK_F16 ? 64 : 128));
}

// own_ws false: ws / cnt are left for the caller to point at shared buffers
// of at least ws_floats / cnt_ints elements (zeroed)
int matrix_alloc(Matrix* m, int src_quant, int rows, int cols, cudaStream_t s, bool own_ws = true);
// the GEMM's TMA maps of a q4_0 / q8_0 matrix (tn_gemm.cu); false if the driver cannot encode them
bool gemm_encode_maps(Matrix* m);
// launch shape of the tensor-core matvec of a q4_0 / q8_0 matrix (at allocation)
int mm_prepare(Matrix* m);
// Repack src_rows rows of a packed tensor (device memory, reference layout,
// `cols` columns) into rows dst_off + r * dst_stride of m.
int matrix_repack(Matrix* m, const uint8_t* d_src, int src_quant, int src_rows, int dst_off,
                  int dst_stride, cudaStream_t s);
void matrix_free(Matrix* m);
int matrix_dequant(const Matrix& m, float* out, cudaStream_t s);

enum EpiMode { EPI_STORE = 0, EPI_RESID = 1, EPI_SWIGLU = 2, EPI_QKV_ROPE = 3 };
// y = W x for T tokens.  STORE: y[t*ldy + r] = v.  RESID: y[t*ldy + r] += v.
// SWIGLU: rows (2i, 2i+1) hold (gate_i, up_i); y[t*ldy + i] = silu(gate) * up.
// err: device int set to 1 if a bounded wait inside a kernel gave up.
// q4_0 / q8_0 matrices take the tensor-core dequant-GEMM from kGemmMinTokens
// tokens on when `gemm_scratch` (gemm_scratch_bytes(T, cols) bytes) is given.
int matvec(const Matrix& m, int T, const float* x, int ldx, float* y, int ldy, int mode, int* err,
           void* gemm_scratch, size_t gemm_scratch_bytes, cudaStream_t s);

// ---- tcgen05 dequant-GEMM (tn_gemm.cu) for steps of many tokens
// (below this the decode matvec, two tokens per launch, streams the weights
// faster than the GEMM dequantises them: measured crossover near 14 tokens)
constexpr int kGemmMinTokens = 16;
bool gemm_ok(const Matrix& m, int T);
// N tiling of T tokens: ntiles tiles of NT tokens (NT a multiple of 16, <= 128)
void gemm_tiling(int T, int* NT, int* ntiles);
// scratch of a T-token GEMM over `cols` columns: the prepared fp16 hi / lo
// activation tiles and the per-token scales
size_t gemm_scratch_bytes(int T, int cols);
// byte offset of the split-K arrival counters in that scratch: zero them when
// the scratch is allocated (every launch leaves them at zero)
size_t gemm_counter_offset(int T, int cols);
// y = W x (rows of x at rowsel[t] if given) with a STORE / RESID / SWIGLU epilogue
int gemm(const Matrix& m, int T, const float* x, int ldx, const int* rowsel, float* y, int ldy, int mode,
         void* scratch, size_t scratch_bytes, int* err, cudaStream_t s);

// Element type of a KV cache: f32 (the reference's rows) or, opt-in, fp16 or
// fp8 e4m3 (rounded to nearest even when appended; e4m3 saturates at +-448
// and carries no scale).
enum KvType { KV_F32 = 0, KV_F16 = 1, KV_F8 = 2 };
__host__ __device__ constexpr size_t kv_elem_bytes(int kv_type) {
  return kv_type == KV_F16 ? 2 : (kv_type == KV_F8 ? 1 : 4);
}
__device__ __forceinline__ void kv_store(void* base, size_t i, int kv_type, float v) {
  if (kv_type == KV_F16) reinterpret_cast<__half*>(base)[i] = __float2half_rn(v);
  else if (kv_type == KV_F8) reinterpret_cast<__nv_fp8_e4m3*>(base)[i] = __nv_fp8_e4m3(v);
  else reinterpret_cast<float*>(base)[i] = v;
}

// per-row bookkeeping of a step: KV slot, RoPE position, KV write index, attention length
struct RowInfo {
  int slot, pos, kv_idx, len;
};

// Where a sequence's KV rows live, in elements from the cache base pointer
// (a layer's K or V).  Contiguous: row i of sequence slot s at
// s * slot_stride + kvh * kvh_stride + i * hd.  Paged: the row is row
// i & (2^shift - 1) of page pages[s * max_pages + (i >> shift)], a page at
// page * slot_stride with kvh_stride between its KV heads.
struct KvMap {
  size_t slot_stride = 0, kvh_stride = 0;
  const int* pages = nullptr;  // [slot][max_pages] page ids (paged), else null
  int max_pages = 0, shift = 0;
};
__device__ __forceinline__ size_t kv_row_off(const KvMap& m, int slot, int kvh, int i, int hd) {
  if (m.pages == nullptr) return (size_t)slot * m.slot_stride + (size_t)kvh * m.kvh_stride + (size_t)i * hd;
  const int pg = m.pages[(size_t)slot * m.max_pages + (i >> m.shift)];
  return (size_t)pg * m.slot_stride + (size_t)kvh * m.kvh_stride + (size_t)(i & ((1 << m.shift) - 1)) * hd;
}

int rmsnorm(const float* h, int ldh, const int* rowsel, const float* w, float* out, int ldo, int H,
            int T, cudaStream_t s);

// Fusions of the decode matvec (matvec_dec):
//   prologue: x rows are the raw hidden state (row t at rowsel[t] if given),
//             normalised in the kernel with RMSNorm weights norm_w;
//   EPI_QKV_ROPE: rows [0, q_dim) and [q_dim, q_dim + kv_dim) hold q and k in
//             RoPE pair-interleaved order; the epilogue rotates each pair
//             (cos/sin table cs) and writes q_out and the K cache, and writes
//             the V rows to the V cache, at each token's RowInfo slot / index.
struct MvFuse {
  const float* norm_w = nullptr;
  const int* rowsel = nullptr;
  const RowInfo* rinfo = nullptr;
  const double2* cs = nullptr;
  float* q_out = nullptr;
  void* kc = nullptr;  // kv_type elements
  void* vc = nullptr;
  int kv_type = KV_F32;
  KvMap kv;
  int q_dim = 0, kv_dim = 0, hd = 0;
};
// the fused decode matvec handles q4_0 / q8_0 matrices; tokens are taken two at a time
bool matvec_dec_ok(const Matrix& m, int T);
// err: device int set to 1 if a bounded wait inside the kernel gave up
int matvec_dec(const Matrix& m, int T, const float* x, int ldx, float* y, int ldy, int mode, const MvFuse& f,
               int* err, cudaStream_t s);
// zero the split-K counters and workspace (after a launch gave up part way)
void matrix_reset_counters(const Matrix& m, cudaStream_t s);
int embed_rows(const Matrix& emb, const int* ids, int T, float* out, int ldo, int* d_err,
               cudaStream_t s);
int rope_table(const RowInfo* rows, const double* freq, int half, int T, double2* cs, cudaStream_t s);
int rope_kv(const float* qkv, int ldqkv, const RowInfo* rows, const double2* cs, float* q_out,
            void* kc, void* vc, int kv_type, const KvMap& kv, int nH, int nKV, int hd, int T, cudaStream_t s);

// One-query GQA attention (web/inference-worker.js:556-564) for T rows, one
// kernel (tn_attn.cu): CTA (split, KV head, row) over its share of the row's
// positions; several splits merge in split order, within a thread-block
// cluster (up to 8) or through a workspace (the last CTA of a (row, KV head)).
struct AttnPlan {
  int splits = 1;
  bool cluster = false;  // the splits merge within a thread-block cluster
  size_t ws_floats = 0;  // partials of the split rows
  size_t cnt_ints = 0;   // arrival counters, zero between launches
};
// splits for T rows over caches of up to max_ctx positions; a workspace of at
// most ws_cap_floats floats bounds them
AttnPlan attn_plan(int T, int nH, int nKV, int hd, int max_ctx, int kv_type, size_t ws_cap_floats = SIZE_MAX);
// kc / vc: kv_type elements.  A paged map may give each CTA at most
// kAttnMaxPages pages: ceil(max_ctx / page positions) + 1 <= kAttnMaxPages.
constexpr int kAttnMaxPages = 1024;
int attention(const float* q, int ldq, const void* kc, const void* vc, int kv_type, const KvMap& kv,
              const RowInfo* rows, int T, int nH, int nKV, int hd, const AttnPlan& plan, float* out, int ldo,
              float* ws, int* cnt, cudaStream_t s);

int hop_encode_rows(const float* h, int ldh, const int* rowsel, int T, int H, uint16_t* out,
                    cudaStream_t s);
int hop_decode(const uint16_t* in, uint64_t n, float* out, cudaStream_t s);
int hop_encode_flat(const float* in, uint64_t n, uint16_t* out, cudaStream_t s);
double sample_uniform(uint64_t seed, uint64_t row);

// sampler parameters live in device memory (a captured graph stays valid):
// d_params[3 r .. 3 r + 2] = temperature, top_p, uniform draw of row r
int sample_rows(float* logits, int n_rows, int vocab, const double* d_params, int* out,
                cudaStream_t s);

int num_sms();

}  // namespace tn
