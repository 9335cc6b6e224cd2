// tn_abi.cu -- single-op C entry points: quantised matrices, attention, the
// activation hop codec and the sampler, for parity tests and microbenchmarks.
#include <mutex>
#include <vector>

#include "tn_kernels.cuh"
#include "tn_ptx.cuh"

namespace tn {

struct DevSwitch {
  int prev = -1;
  cudaError_t err = cudaSuccess;
  explicit DevSwitch(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) err = cudaSetDevice(dev);
  }
  ~DevSwitch() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

// the row table of tn_attention's rows; also zeroes the split arrival counters
__global__ void k_rows_from_slots(const int32_t* __restrict__ slot, const int32_t* __restrict__ len, int n,
                                  int n_slots, int max_ctx, RowInfo* __restrict__ rows, int* __restrict__ cnt,
                                  int n_cnt) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  for (int i = r; i < n_cnt; i += gridDim.x * blockDim.x) cnt[i] = 0;
  if (r >= n) return;
  int s = slot[r], l = len[r];
  if (s < 0 || s >= n_slots || l < 1) {
    s = 0;
    l = 0;
  }
  rows[r] = RowInfo{s, 0, 0, l > max_ctx ? max_ctx : l};
}

// the row table of tn_attention_paged's rows (row r reads page-table row r);
// a row whose used page ids leave [0, n_pages) gets no positions
__global__ void k_rows_from_pages(const int32_t* __restrict__ pages, const int32_t* __restrict__ len, int n,
                                  int max_pages, int shift, int n_pages, RowInfo* __restrict__ rows,
                                  int* __restrict__ cnt, int n_cnt) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  for (int i = r; i < n_cnt; i += gridDim.x * blockDim.x) cnt[i] = 0;
  if (r >= n) return;
  const int max_ctx = max_pages << shift;
  int l = len[r];
  l = l < 1 ? 0 : (l > max_ctx ? max_ctx : l);
  const int used = (l + (1 << shift) - 1) >> shift;
  for (int j = 0; j < used; j++) {
    const int pg = pages[(size_t)r * max_pages + j];
    if (pg < 0 || pg >= n_pages) l = 0;
  }
  rows[r] = RowInfo{r, 0, 0, l};
}

// The kernels' bounded mbarrier wait (mbar_wait) on a barrier that no thread
// arrives at, with a limit of `limit` cycles: the wait gives up, the CTA's
// abort flag is raised, and the status says so -- the path a real kernel takes
// when its copy pipeline stalls, made to run out on purpose without a fault.
static __device__ int g_wait_probe_status;
__global__ void k_wait_probe(long long limit) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ volatile int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const bool ok = mbar_wait(&bar, 0, &abort_flag, limit);
  __syncthreads();
  if (threadIdx.x == 0) g_wait_probe_status = ok && !abort_flag ? 0 : 1;
}

}  // namespace tn

using namespace tn;

extern "C" int tn_test_bounded_wait(uint64_t limit_cycles) {
  clear_error();
  TN_REQUIRE(limit_cycles > 0 && limit_cycles <= (uint64_t)kWaitLimitCycles, TN_EINVAL,
             "tn_test_bounded_wait: limit of %llu cycles", (unsigned long long)limit_cycles);
  int st = -1;
  TN_CHECK_CUDA(cudaMemcpyToSymbol(g_wait_probe_status, &st, sizeof(int)));
  k_wait_probe<<<1, 64>>>((long long)limit_cycles);
  TN_CHECK_LAUNCH();
  TN_CHECK_CUDA(cudaDeviceSynchronize());
  TN_CHECK_CUDA(cudaMemcpyFromSymbol(&st, g_wait_probe_status, sizeof(int)));
  TN_REQUIRE(st == 0 || st == 1, TN_ECUDA, "tn_test_bounded_wait: status %d", st);
  if (st) {
    set_error("bounded wait gave up after %llu cycles", (unsigned long long)limit_cycles);
    return TN_ETIMEOUT;
  }
  return TN_OK;
}

struct tn_matrix {
  Matrix m;
  int device = 0;
  int* d_err = nullptr;  // bounded-wait flag of the decode kernel
  // activation tiles of the dequant-GEMM, grown on first use by a token count
  void* gemm_scratch = nullptr;
  size_t gemm_bytes = 0;
};

extern "C" int tn_matrix_create(int32_t device, int32_t quant, int32_t rows, int32_t cols, const void* packed,
                                uint64_t len, int32_t on_device, tn_matrix** out) {
  clear_error();
  TN_REQUIRE(out && packed && rows > 0 && cols > 0, TN_EINVAL, "tn_matrix_create: bad argument");
  *out = nullptr;
  const uint64_t need = quant_bytes((uint64_t)rows * cols, quant);
  TN_REQUIRE(need != 0, TN_EUNSUPPORTED, "unsupported quant %d", quant);
  TN_REQUIRE(len >= need, TN_EINVAL, "tn_matrix_create: %llu bytes given, %llu needed",
             (unsigned long long)len, (unsigned long long)need);
  TN_REQUIRE(cols <= 32768, TN_EUNSUPPORTED, "tn_matrix_create: more than 32768 columns");
  DevSwitch g(device);
  TN_REQUIRE(g.err == cudaSuccess, TN_ECUDA, "cudaSetDevice(%d): %s", device, cudaGetErrorString(g.err));
  tn_matrix* M = new (std::nothrow) tn_matrix();
  TN_REQUIRE(M, TN_ENOMEM, "out of host memory");
  M->device = device;
  int rc = matrix_alloc(&M->m, quant, rows, cols, 0);
  if (!rc && (cudaMalloc(&M->d_err, sizeof(int)) != cudaSuccess || cudaMemset(M->d_err, 0, sizeof(int)) != cudaSuccess)) {
    set_error("tn_matrix_create: error flag allocation failed");
    rc = TN_ENOMEM;
  }
  uint8_t* staging = nullptr;
  const uint8_t* src = (const uint8_t*)packed;
  if (!rc && !on_device) {
    if (cudaMalloc(&staging, need) != cudaSuccess ||
        cudaMemcpy(staging, packed, need, cudaMemcpyHostToDevice) != cudaSuccess) {
      set_error("tn_matrix_create: staging upload failed");
      rc = TN_ECUDA;
    }
    src = staging;
  }
  if (!rc) rc = matrix_repack(&M->m, src, quant, rows, 0, 1, 0);
  if (!rc && cudaStreamSynchronize(0) != cudaSuccess) {
    set_error("tn_matrix_create: repack failed");
    rc = TN_ECUDA;
  }
  if (staging) cudaFree(staging);
  if (rc) {
    matrix_free(&M->m);
    if (M->d_err) cudaFree(M->d_err);
    delete M;
    return rc;
  }
  *out = M;
  return TN_OK;
}

extern "C" int tn_matrix_matvec(const tn_matrix* m, int32_t n_tokens, const float* d_x, float* d_y,
                                void* stream) {
  clear_error();
  TN_REQUIRE(m && d_x && d_y && n_tokens >= 0, TN_EINVAL, "tn_matrix_matvec: bad argument");
  DevSwitch g(m->device);
  tn_matrix* mm = const_cast<tn_matrix*>(m);
  if (gemm_ok(m->m, n_tokens)) {
    const size_t need = gemm_scratch_bytes(n_tokens, m->m.cols);
    if (need > mm->gemm_bytes) {
      // (the first call with more tokens than any before allocates; later ones reuse)
      TN_CHECK_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
      if (mm->gemm_scratch) cudaFree(mm->gemm_scratch);
      mm->gemm_scratch = nullptr;
      mm->gemm_bytes = 0;
      TN_CHECK_CUDA(cudaMalloc(&mm->gemm_scratch, need));
      mm->gemm_bytes = need;
      TN_CHECK_CUDA(cudaMemset(mm->gemm_scratch, 0, need));  // the split-K counters start at zero
    }
  }
  return matvec(m->m, n_tokens, d_x, m->m.cols, d_y, m->m.rows, EPI_STORE, m->d_err, mm->gemm_scratch,
                mm->gemm_bytes, (cudaStream_t)stream);
}

extern "C" int tn_matrix_dequant(const tn_matrix* m, float* d_out, void* stream) {
  clear_error();
  TN_REQUIRE(m && d_out, TN_EINVAL, "tn_matrix_dequant: bad argument");
  DevSwitch g(m->device);
  return matrix_dequant(m->m, d_out, (cudaStream_t)stream);
}

extern "C" uint64_t tn_matrix_device_bytes(const tn_matrix* m) { return m ? m->m.bytes : 0; }

extern "C" int tn_matrix_counter_sum(const tn_matrix* m, int64_t* out) {
  clear_error();
  TN_REQUIRE(m && out, TN_EINVAL, "tn_matrix_counter_sum: bad argument");
  DevSwitch g(m->device);
  *out = 0;
  if (!m->m.cnt || !m->m.cnt_ints) return TN_OK;
  std::vector<int> h(m->m.cnt_ints);
  TN_CHECK_CUDA(cudaDeviceSynchronize());
  TN_CHECK_CUDA(cudaMemcpy(h.data(), m->m.cnt, h.size() * sizeof(int), cudaMemcpyDeviceToHost));
  for (int v : h) *out += v;
  return TN_OK;
}

extern "C" void tn_matrix_free(tn_matrix* m) {
  if (!m) return;
  DevSwitch g(m->device);
  matrix_free(&m->m);
  if (m->d_err) cudaFree(m->d_err);
  if (m->gemm_scratch) cudaFree(m->gemm_scratch);
  delete m;
}

// caller scratch: the row table (the splits merge on chip)
// tn_attention's scratch: the row table (16 bytes a row), the split arrival
// counters and the split partials, each 256-byte aligned
struct AttnScratch {
  AttnPlan plan;
  size_t cnt_off = 0, ws_off = 0, total = 0;
};
static size_t al256(size_t x) { return (x + 255) & ~(size_t)255; }
static AttnScratch attn_scratch(int n_rows, int nH, int nKV, int hd, int max_ctx, int kv_type,
                                size_t cap = SIZE_MAX) {
  AttnScratch a;
  a.cnt_off = al256((size_t)n_rows * sizeof(RowInfo));
  const size_t cnt_bytes = al256((size_t)n_rows * std::max(1, nKV) * sizeof(int));
  a.ws_off = a.cnt_off + cnt_bytes;
  const size_t room = cap > a.ws_off ? (cap - a.ws_off) / sizeof(float) : 0;
  a.plan = attn_plan(n_rows, nH, nKV, hd, max_ctx, kv_type, room);
  a.total = a.plan.splits > 1 ? a.ws_off + al256(a.plan.ws_floats * sizeof(float)) : a.cnt_off;
  return a;
}

// row table (and zeroed split counters), then the one-kernel attention
static int attn_run(int n_rows, int n_slots, int n_heads, int n_kv_heads, int head_dim, int max_ctx, const float* d_q,
                    const void* d_k, const void* d_v, int kv_type, const int32_t* d_slot, const int32_t* d_len,
                    float* d_out, void* scratch, size_t scratch_bytes, cudaStream_t s) {
  const AttnScratch sc = attn_scratch(n_rows, n_heads, n_kv_heads, head_dim, max_ctx, kv_type, scratch_bytes);
  TN_REQUIRE(sc.total <= scratch_bytes, TN_EINVAL, "attention: scratch of %zu bytes, %zu needed", scratch_bytes,
             sc.total);
  char* base = (char*)scratch;
  RowInfo* rows = (RowInfo*)base;
  int* cnt = sc.plan.splits > 1 ? (int*)(base + sc.cnt_off) : nullptr;
  float* ws = sc.plan.splits > 1 ? (float*)(base + sc.ws_off) : nullptr;
  const int n_cnt = cnt ? (int)sc.plan.cnt_ints : 0;
  const int work = std::max(n_rows, n_cnt);
  k_rows_from_slots<<<(work + 127) / 128, 128, 0, s>>>(d_slot, d_len, n_rows, n_slots, max_ctx, rows, cnt, n_cnt);
  TN_CHECK_LAUNCH();
  KvMap kv;
  kv.kvh_stride = (size_t)max_ctx * head_dim;
  kv.slot_stride = kv.kvh_stride * n_kv_heads;
  return attention(d_q, n_heads * head_dim, d_k, d_v, kv_type, kv, rows, n_rows, n_heads, n_kv_heads, head_dim,
                   sc.plan, d_out, n_heads * head_dim, ws, cnt, s);
}

static int attn_check(const char* fn, int32_t n_rows, int32_t n_slots, int32_t n_heads, int32_t n_kv_heads,
                      int32_t head_dim, int32_t max_ctx, const void* d_q, const void* d_k, const void* d_v,
                      const int32_t* d_slot, const int32_t* d_len, const float* d_out) {
  TN_REQUIRE(n_rows >= 0 && n_slots > 0 && n_heads > 0 && n_kv_heads > 0 && max_ctx > 0, TN_EINVAL,
             "%s: bad sizes", fn);
  TN_REQUIRE(d_q && d_k && d_v && d_slot && d_len && d_out, TN_EINVAL, "%s: null pointer", fn);
  TN_REQUIRE(head_dim == 32 || head_dim == 64 || head_dim == 128, TN_EUNSUPPORTED, "%s: head_dim %d unsupported",
             fn, head_dim);
  return TN_OK;
}

extern "C" uint64_t tn_attention_scratch_bytes(int32_t n_rows, int32_t n_heads, int32_t n_kv_heads,
                                               int32_t head_dim, int32_t max_ctx) {
  if (n_rows <= 0 || n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0 || max_ctx <= 0) return 0;
  // (enough for every cache element type)
  return std::max({attn_scratch(n_rows, n_heads, n_kv_heads, head_dim, max_ctx, KV_F32).total,
                   attn_scratch(n_rows, n_heads, n_kv_heads, head_dim, max_ctx, KV_F16).total,
                   attn_scratch(n_rows, n_heads, n_kv_heads, head_dim, max_ctx, KV_F8).total});
}

static int attn_entry(const char* fn, int kv_type, int32_t n_rows, int32_t n_slots, int32_t n_heads,
                      int32_t n_kv_heads, int32_t head_dim, int32_t max_ctx, const float* d_q, const void* d_k,
                      const void* d_v, const int32_t* d_slot, const int32_t* d_len, float* d_out, void* d_scratch,
                      uint64_t scratch_bytes, void* stream) {
  clear_error();
  int rc = attn_check(fn, n_rows, n_slots, n_heads, n_kv_heads, head_dim, max_ctx, d_q, d_k, d_v, d_slot, d_len,
                      d_out);
  if (rc) return rc;
  TN_REQUIRE(d_scratch, TN_EINVAL, "%s: null scratch", fn);
  TN_REQUIRE((reinterpret_cast<uintptr_t>(d_scratch) & 255) == 0, TN_EINVAL, "%s: scratch must be 256-byte aligned",
             fn);
  if (n_rows == 0) return TN_OK;
  return attn_run(n_rows, n_slots, n_heads, n_kv_heads, head_dim, max_ctx, d_q, d_k, d_v, kv_type, d_slot, d_len,
                  d_out, d_scratch, scratch_bytes, (cudaStream_t)stream);
}

extern "C" int tn_attention(int32_t n_rows, int32_t n_slots, int32_t n_heads, int32_t n_kv_heads,
                            int32_t head_dim, int32_t max_ctx, const float* d_q, const float* d_k,
                            const float* d_v, const int32_t* d_slot, const int32_t* d_len, float* d_out,
                            void* d_scratch, uint64_t scratch_bytes, void* stream) {
  return attn_entry("tn_attention", KV_F32, n_rows, n_slots, n_heads, n_kv_heads, head_dim, max_ctx, d_q, d_k, d_v,
                    d_slot, d_len, d_out, d_scratch, scratch_bytes, stream);
}

extern "C" int tn_attention_f8(int32_t n_rows, int32_t n_slots, int32_t n_heads, int32_t n_kv_heads,
                               int32_t head_dim, int32_t max_ctx, const float* d_q, const uint8_t* d_k,
                               const uint8_t* d_v, const int32_t* d_slot, const int32_t* d_len, float* d_out,
                               void* d_scratch, uint64_t scratch_bytes, void* stream) {
  return attn_entry("tn_attention_f8", KV_F8, n_rows, n_slots, n_heads, n_kv_heads, head_dim, max_ctx, d_q, d_k,
                    d_v, d_slot, d_len, d_out, d_scratch, scratch_bytes, stream);
}

extern "C" int tn_attention_f16(int32_t n_rows, int32_t n_slots, int32_t n_heads, int32_t n_kv_heads,
                                int32_t head_dim, int32_t max_ctx, const float* d_q, const uint16_t* d_k,
                                const uint16_t* d_v, const int32_t* d_slot, const int32_t* d_len, float* d_out,
                                void* d_scratch, uint64_t scratch_bytes, void* stream) {
  return attn_entry("tn_attention_f16", KV_F16, n_rows, n_slots, n_heads, n_kv_heads, head_dim, max_ctx, d_q, d_k,
                    d_v, d_slot, d_len, d_out, d_scratch, scratch_bytes, stream);
}

extern "C" int tn_attention_paged(int32_t kv_type, int32_t n_rows, int32_t n_heads, int32_t n_kv_heads,
                                  int32_t head_dim, int32_t page_tokens, int32_t max_pages, int32_t n_pages,
                                  const float* d_q, const void* d_k, const void* d_v, const int32_t* d_pages,
                                  const int32_t* d_len, float* d_out, void* d_scratch, uint64_t scratch_bytes,
                                  void* stream) {
  clear_error();
  TN_REQUIRE(kv_type == KV_F32 || kv_type == KV_F16 || kv_type == KV_F8, TN_EINVAL,
             "tn_attention_paged: kv_type %d", kv_type);
  TN_REQUIRE(page_tokens >= 16 && page_tokens <= 4096 && (page_tokens & (page_tokens - 1)) == 0, TN_EINVAL,
             "tn_attention_paged: page_tokens %d (a power of two in [16, 4096])", page_tokens);
  TN_REQUIRE(max_pages > 0 && max_pages + 1 <= kAttnMaxPages && n_pages > 0, TN_EINVAL,
             "tn_attention_paged: max_pages %d (1 .. %d), n_pages %d", max_pages, kAttnMaxPages - 1, n_pages);
  const int max_ctx = max_pages * page_tokens;
  int rc = attn_check("tn_attention_paged", n_rows, 1, n_heads, n_kv_heads, head_dim, max_ctx, d_q, d_k, d_v,
                      d_pages, d_len, d_out);
  if (rc) return rc;
  TN_REQUIRE(d_scratch, TN_EINVAL, "tn_attention_paged: null scratch");
  TN_REQUIRE((reinterpret_cast<uintptr_t>(d_scratch) & 255) == 0, TN_EINVAL,
             "tn_attention_paged: scratch must be 256-byte aligned");
  if (n_rows == 0) return TN_OK;
  const AttnScratch sc = attn_scratch(n_rows, n_heads, n_kv_heads, head_dim, max_ctx, kv_type, scratch_bytes);
  TN_REQUIRE(sc.total <= scratch_bytes, TN_EINVAL, "attention: scratch of %llu bytes, %zu needed",
             (unsigned long long)scratch_bytes, sc.total);
  int shift = 0;
  while ((1 << shift) < page_tokens) shift++;
  char* base = (char*)d_scratch;
  RowInfo* rows = (RowInfo*)base;
  int* cnt = sc.plan.splits > 1 ? (int*)(base + sc.cnt_off) : nullptr;
  float* ws = sc.plan.splits > 1 ? (float*)(base + sc.ws_off) : nullptr;
  const int n_cnt = cnt ? (int)sc.plan.cnt_ints : 0;
  const int work = std::max((int)n_rows, n_cnt);
  const cudaStream_t s = (cudaStream_t)stream;
  k_rows_from_pages<<<(work + 127) / 128, 128, 0, s>>>(d_pages, d_len, n_rows, max_pages, shift, n_pages, rows, cnt,
                                                       n_cnt);
  TN_CHECK_LAUNCH();
  KvMap kv;
  kv.kvh_stride = (size_t)page_tokens * head_dim;
  kv.slot_stride = kv.kvh_stride * n_kv_heads;
  kv.pages = d_pages;
  kv.max_pages = max_pages;
  kv.shift = shift;
  return attention(d_q, n_heads * head_dim, d_k, d_v, kv_type, kv, rows, n_rows, n_heads, n_kv_heads, head_dim,
                   sc.plan, d_out, n_heads * head_dim, ws, cnt, s);
}

// ---- tn_attention_static: attention with its scratch in a fixed device array,
// for callers that cannot allocate device memory (see tabnet_stage.h).
static __device__ __align__(256) unsigned char g_attn_static_scratch[TN_ATTENTION_STATIC_SCRATCH_BYTES];

namespace tn {
constexpr int kMaxStaticDevices = 64;
static std::mutex g_attn_static_mu;
static void* g_attn_static_ptr[kMaxStaticDevices];  // this array's device address, per device

// Host code cannot use g_attn_static_scratch as a pointer (on the host it names
// a stand-in, not device memory): look the address up for the current device,
// once per device, with that device current.
static int attn_static_scratch(void** out) {
  int dev = -1;
  TN_CHECK_CUDA(cudaGetDevice(&dev));
  TN_REQUIRE(dev >= 0 && dev < kMaxStaticDevices, TN_EUNSUPPORTED, "tn_attention_static: device %d", dev);
  std::lock_guard<std::mutex> lk(g_attn_static_mu);
  if (!g_attn_static_ptr[dev]) {
    void* p = nullptr;
    TN_CHECK_CUDA(cudaGetSymbolAddress(&p, g_attn_static_scratch));
    g_attn_static_ptr[dev] = p;
  }
  *out = g_attn_static_ptr[dev];
  return TN_OK;
}
}  // namespace tn

extern "C" int tn_attention_static(int32_t n_rows, int32_t n_slots, int32_t n_heads, int32_t n_kv_heads,
                                   int32_t head_dim, int32_t max_ctx, const float* d_q, const float* d_k,
                                   const float* d_v, const int32_t* d_slot, const int32_t* d_len, float* d_out,
                                   void* stream) {
  clear_error();
  int rc = attn_check("tn_attention_static", n_rows, n_slots, n_heads, n_kv_heads, head_dim, max_ctx, d_q, d_k, d_v,
                      d_slot, d_len, d_out);
  if (rc) return rc;
  if (n_rows == 0) return TN_OK;
  // the split count is bounded so that the partials fit the fixed array
  const size_t need = attn_scratch(n_rows, n_heads, n_kv_heads, head_dim, max_ctx, KV_F32,
                                   TN_ATTENTION_STATIC_SCRATCH_BYTES).total;
  TN_REQUIRE(need <= TN_ATTENTION_STATIC_SCRATCH_BYTES, TN_ECAPACITY,
             "tn_attention_static: %d rows need %zu bytes of scratch, above the fixed %u; "
             "use tn_attention with caller scratch",
             n_rows, need, (unsigned)TN_ATTENTION_STATIC_SCRATCH_BYTES);
  void* scratch = nullptr;
  rc = attn_static_scratch(&scratch);
  if (rc) return rc;
  return attn_run(n_rows, n_slots, n_heads, n_kv_heads, head_dim, max_ctx, d_q, d_k, d_v, KV_F32, d_slot, d_len,
                  d_out, scratch, TN_ATTENTION_STATIC_SCRATCH_BYTES, (cudaStream_t)stream);
}

extern "C" int tn_hop_encode(const float* d_in, uint16_t* d_out, uint64_t n, void* stream) {
  clear_error();
  TN_REQUIRE(n == 0 || (d_in && d_out), TN_EINVAL, "tn_hop_encode: null pointer");
  return hop_encode_flat(d_in, n, d_out, (cudaStream_t)stream);
}

extern "C" int tn_hop_decode(const uint16_t* d_in, float* d_out, uint64_t n, void* stream) {
  clear_error();
  TN_REQUIRE(n == 0 || (d_in && d_out), TN_EINVAL, "tn_hop_decode: null pointer");
  return hop_decode(d_in, n, d_out, (cudaStream_t)stream);
}

extern "C" uint16_t tn_hop_encode_host(float v) { return hop_encode(v); }

extern "C" double tn_sample_uniform(uint64_t rng_seed, uint64_t row) { return sample_uniform(rng_seed, row); }

extern "C" int tn_sample(float* d_logits, int32_t n_rows, int32_t vocab, double temperature, double top_p,
                         uint64_t rng_seed, int32_t* d_out, void* stream) {
  clear_error();
  TN_REQUIRE(d_logits && d_out && n_rows >= 0 && vocab > 0, TN_EINVAL, "tn_sample: bad argument");
  if (n_rows == 0) return TN_OK;
  std::vector<double> p(3 * (size_t)n_rows);
  for (int r = 0; r < n_rows; r++) {
    p[3 * r] = temperature;
    p[3 * r + 1] = top_p;
    p[3 * r + 2] = sample_uniform(rng_seed, (uint64_t)r);
  }
  double* dp = nullptr;
  TN_CHECK_CUDA(cudaMalloc(&dp, p.size() * sizeof(double)));
  cudaStream_t s = (cudaStream_t)stream;
  int rc = TN_OK;
  if (cudaMemcpyAsync(dp, p.data(), p.size() * sizeof(double), cudaMemcpyHostToDevice, s) != cudaSuccess) {
    set_error("tn_sample: parameter upload failed");
    rc = TN_ECUDA;
  }
  // the sampler overwrites logits with probabilities when temperature > 0
  if (!rc) rc = sample_rows(d_logits, n_rows, vocab, dp, d_out, s);
  if (cudaStreamSynchronize(s) != cudaSuccess && !rc) {
    set_error("tn_sample: %s", cudaGetErrorString(cudaGetLastError()));
    rc = TN_ECUDA;
  }
  cudaFree(dp);
  return rc;
}
