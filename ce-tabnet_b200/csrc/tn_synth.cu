// tn_synth.cu -- seeded synthetic model packs in the reference byte layout.
//
// The reference ships no quantiser and no runnable model pack
// (tools/shard-model.js:5-7, models/README.md:52-53), so benchmarks and parity
// tests build their own: per-layer buffers in layerLayout order
// (web/inference-worker.js:142-159) with q4_0 / q8_0 blocks as dequantToF32
// reads them (:102-129).  The generator (tn_common.cuh) is integer hashing plus
// IEEE single operations, so the host writer and the device writer produce the
// same bytes; big packs are written directly in device memory.
#include <algorithm>
#include <cmath>
#include <functional>
#include <thread>
#include <vector>

#include "tn_common.cuh"

namespace tn {

enum { SYN_MATRIX = 0, SYN_NORM = 1 };

__global__ void k_synth_blocks(uint64_t key, uint64_t count, int quant, uint8_t* out) {
  const uint64_t nb = (count + 31ull) / 32ull;
  const uint64_t bb = quant == TN_QUANT_Q8_0 ? 34ull : 18ull;
  for (uint64_t b = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; b < nb;
       b += (uint64_t)gridDim.x * blockDim.x)
    synth_quant_block(key, count, b, quant, out + b * bb);
}

__host__ __device__ inline void synth_plain_elem(uint64_t key, uint64_t i, int quant, int role,
                                                 uint8_t* out) {
  float v = synth_value(key, i);
  if (role == SYN_NORM) v = fadd_rn(1.0f, v);
  if (quant == TN_QUANT_F32) {
    const uint32_t u = f2u(v);
    for (int k = 0; k < 4; k++) out[i * 4 + k] = (uint8_t)(u >> (8 * k));
  } else {
    const uint16_t h = f32_to_f16_rne(v);
    out[i * 2] = (uint8_t)(h & 0xff);
    out[i * 2 + 1] = (uint8_t)(h >> 8);
  }
}

__global__ void k_synth_plain(uint64_t key, uint64_t count, int quant, int role, uint8_t* out) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count;
       i += (uint64_t)gridDim.x * blockDim.x)
    synth_plain_elem(key, i, quant, role, out);
}

static void host_parallel(uint64_t n, const std::function<void(uint64_t, uint64_t)>& fn) {
  unsigned nt = std::thread::hardware_concurrency();
  if (nt == 0) nt = 1;
  if (n < 4096 || nt == 1) {
    fn(0, n);
    return;
  }
  if (nt > 64) nt = 64;
  std::vector<std::thread> th;
  for (unsigned t = 0; t < nt; t++) {
    const uint64_t a = n * t / nt, b = n * (t + 1) / nt;
    th.emplace_back([&fn, a, b] { fn(a, b); });
  }
  for (auto& x : th) x.join();
}

// one tensor of `count` elements in `quant` at `out`
static int synth_tensor_impl(uint64_t key, uint64_t count, int quant, int role, uint8_t* out,
                             bool on_device, cudaStream_t stream) {
  if (quant == TN_QUANT_Q4_0 || quant == TN_QUANT_Q8_0) {
    TN_REQUIRE(role == SYN_MATRIX, TN_EINVAL, "norm tensors are stored f16");
    const uint64_t nb = (count + 31ull) / 32ull, bb = quant == TN_QUANT_Q8_0 ? 34ull : 18ull;
    if (on_device) {
      const unsigned grid = (unsigned)std::min<uint64_t>((nb + 255) / 256, 148ull * 64ull);
      k_synth_blocks<<<grid ? grid : 1, 256, 0, stream>>>(key, count, quant, out);
      TN_CHECK_LAUNCH();
    } else {
      host_parallel(nb, [&](uint64_t a, uint64_t b) {
        for (uint64_t i = a; i < b; i++) synth_quant_block(key, count, i, quant, out + i * bb);
      });
    }
    return TN_OK;
  }
  TN_REQUIRE(quant == TN_QUANT_F32 || quant == TN_QUANT_F16, TN_EUNSUPPORTED, "unsupported quant %d",
             quant);
  if (on_device) {
    const unsigned grid = (unsigned)std::min<uint64_t>((count + 255) / 256, 148ull * 64ull);
    k_synth_plain<<<grid ? grid : 1, 256, 0, stream>>>(key, count, quant, role, out);
    TN_CHECK_LAUNCH();
  } else {
    host_parallel(count, [&](uint64_t a, uint64_t b) {
      for (uint64_t i = a; i < b; i++) synth_plain_elem(key, i, quant, role, out);
    });
  }
  return TN_OK;
}

}  // namespace tn

using namespace tn;

extern "C" uint64_t tn_quant_bytes(uint64_t count, int32_t quant) { return quant_bytes(count, quant); }

extern "C" uint64_t tn_layer_bytes(const tn_dims* d, int32_t quant) {
  if (!d) return 0;
  LayerLayout L;
  if (!layer_layout(d->hidden_dim, d->n_heads, d->n_kv_heads, d->ffn_dim, quant, &L)) return 0;
  return L.total;
}

extern "C" int tn_synth_layer(uint64_t seed, int32_t layer_idx, const tn_dims* d, int32_t quant,
                              void* out, int32_t on_device, void* stream) {
  clear_error();
  TN_REQUIRE(d && out, TN_EINVAL, "tn_synth_layer: null argument");
  LayerLayout L;
  TN_REQUIRE(layer_layout(d->hidden_dim, d->n_heads, d->n_kv_heads, d->ffn_dim, quant, &L),
             TN_EUNSUPPORTED, "tn_synth_layer: bad dims or unsupported quant %d", quant);
  uint8_t* base = (uint8_t*)out;
  for (int t = 0; t < 9; t++) {
    const bool norm = (t == 0 || t == 5);
    const int rc = synth_tensor_impl(synth_key(seed, layer_tag(layer_idx, t)), L.count[t],
                                     norm ? TN_QUANT_F16 : quant, norm ? SYN_NORM : SYN_MATRIX,
                                     base + L.off[t], on_device != 0, (cudaStream_t)stream);
    if (rc) return rc;
  }
  return TN_OK;
}

extern "C" int tn_synth_tensor(uint64_t seed, int32_t tag, const tn_dims* d, int32_t quant, void* out,
                               int32_t on_device, void* stream) {
  clear_error();
  TN_REQUIRE(d && out, TN_EINVAL, "tn_synth_tensor: null argument");
  TN_REQUIRE(tag == TN_TAG_EMBED || tag == TN_TAG_NORM || tag == TN_TAG_LM_HEAD, TN_EINVAL,
             "tn_synth_tensor: unknown tag %d", tag);
  if (tag == TN_TAG_NORM)
    return synth_tensor_impl(synth_key(seed, (uint32_t)tag), (uint64_t)d->hidden_dim, TN_QUANT_F16,
                             SYN_NORM, (uint8_t*)out, on_device != 0, (cudaStream_t)stream);
  const uint64_t count = (uint64_t)d->vocab * (uint64_t)d->hidden_dim;
  return synth_tensor_impl(synth_key(seed, (uint32_t)tag), count, quant, SYN_MATRIX, (uint8_t*)out,
                           on_device != 0, (cudaStream_t)stream);
}
