// tn_kernels.cuh -- device data structures and launchers of the stage engine.
#pragma once

#include "tn_common.cuh"

namespace tn {

// Device layouts of a [rows x cols] weight matrix after the init-time repack.
//   MK_Q4 : data [rows_pad][nb][16 B]  nibbles in reference order (byte j = elems 2j, 2j+1)
//   MK_Q8 : data [rows_pad][nb][32 B]  int8
//   MK_F16: data [rows_pad][cols_pad]  fp16 bits (zero padded)
//   MK_F32: data [rows_pad][cols_pad]  f32 (zero padded); also holds exactly dequantised
//           q4_0/q8_0 tensors whose rows do not start on a block boundary
//   scales (MK_Q4 / MK_Q8): [rows_pad][nb] fp16 bits, so R consecutive rows are
//           one contiguous run of the data plane plus one of the scale plane
//   rows_pad is a multiple of 16.
enum MatKind { MK_Q4 = 0, MK_Q8 = 1, MK_F16 = 2, MK_F32 = 3 };

struct Matrix {
  int kind = MK_F32;
  int rows = 0, cols = 0;
  int rows_pad = 0, cols_pad = 0, nb = 0;
  uint8_t* data = nullptr;
  uint16_t* scales = nullptr;
  size_t bytes = 0;
  int occ[2] = {0, 0};      // resident CTAs per SM of the matvec launch shapes (1 and 2 tokens per tile)
  // decode matvec launch shape: rows per bulk-copied unit, ring depth, bytes
  int mvt_rows = 0, mvt_stages = 0, mvt_smem = 0;
  int mvt_ctas[2] = {1, 1};  // resident CTAs per SM (1 and 2 tokens)
  uint32_t mvt_stage_bytes = 0;
};

// bytes per 32-element block of the data plane
__host__ __device__ constexpr int kind_block_bytes(int k) {
  return k == MK_Q4 ? 16 : (k == MK_Q8 ? 32 : (k == MK_F16 ? 64 : 128));
}

int matrix_alloc(Matrix* m, int src_quant, int rows, int cols, cudaStream_t s);
// Repack src_rows rows of a packed tensor (device memory, reference layout,
// `cols` columns) into rows dst_off + r * dst_stride of m.
int matrix_repack(Matrix* m, const uint8_t* d_src, int src_quant, int src_rows, int dst_off,
                  int dst_stride, cudaStream_t s);
void matrix_free(Matrix* m);
int matrix_dequant(const Matrix& m, float* out, cudaStream_t s);

enum EpiMode { EPI_STORE = 0, EPI_RESID = 1, EPI_SWIGLU = 2, EPI_QKV_ROPE = 3 };
// y = W x for T tokens.  STORE: y[t*ldy + r] = v.  RESID: y[t*ldy + r] += v.
// SWIGLU: rows (2i, 2i+1) hold (gate_i, up_i); y[t*ldy + i] = silu(gate) * up.
int matvec(const Matrix& m, int T, const float* x, int ldx, float* y, int ldy, int mode,
           cudaStream_t s);

// per-row bookkeeping of a step: KV slot, RoPE position, KV write index, attention length
struct RowInfo {
  int slot, pos, kv_idx, len;
};

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
  float* kc = nullptr;
  float* vc = nullptr;
  size_t slot_stride = 0, kvh_stride = 0;
  int q_dim = 0, kv_dim = 0, hd = 0;
};
// the decode matvec handles up to 2 tokens of q4_0 / q8_0 matrices
bool matvec_dec_ok(const Matrix& m, int T);
// err: device int set to 1 if a bounded wait inside the kernel gave up
int matvec_dec(const Matrix& m, int T, const float* x, int ldx, float* y, int ldy, int mode, const MvFuse& f,
               int* err, cudaStream_t s);
// split-K decode attention with the split merge done by the last CTA of each
// (row, KV head); counters: T * nKV ints, zero between calls
int attention_dec(const float* q, int ldq, const float* kc, const float* vc, size_t slot_stride,
                  size_t kvh_stride, const RowInfo* rows, int T, int nH, int nKV, int hd, int n_splits,
                  float* out, int ldo, void* scratch, int* counters, cudaStream_t s);
int embed_rows(const Matrix& emb, const int* ids, int T, float* out, int ldo, int* d_err,
               cudaStream_t s);
int rope_table(const RowInfo* rows, const double* freq, int half, int T, double2* cs, cudaStream_t s);
int rope_kv(const float* qkv, int ldqkv, const RowInfo* rows, const double2* cs, float* q_out,
            float* kc, float* vc, size_t slot_stride, size_t kvh_stride, int nH, int nKV, int hd, int T,
            cudaStream_t s);

int attn_splits(int T, int nKV, int max_ctx);
size_t attn_scratch_bytes(int T, int nH, int hd, int n_splits);
int attention(const float* q, int ldq, const float* kc, const float* vc, size_t slot_stride,
              size_t kvh_stride, const RowInfo* rows, int T, int nH, int nKV, int hd, int n_splits,
              float* out, int ldo, void* scratch, cudaStream_t s);

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
