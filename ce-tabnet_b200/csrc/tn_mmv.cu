// tn_mmv.cu -- tensor-core dequant-matvec of q4_0 / q8_0 matrices (decode).
//
// The matvec of web/inference-worker.js:523-527 / :545-552 / :567-583
// (dequantised weight rows dotted with an f32 activation row), with the
// weights kept in their 4.5 / 8.5-bit form and the products formed by
// mma.sync m16n8k32 s8 x s8 -> s32 tensor-core instructions:
//
//   A (weights): 16 rows x 32 columns per instruction, the columns being 16
//     elements of block 2p and the same 16 elements of block 2p + 1.  A q4_0
//     weight (n - 8) is stored as the 4-bit two's complement n ^ 8, so
//     masking a byte's high nibble (or shifting the low one up) yields
//     16 (n - 8) as an s8 with one LOP3 / SHF per four weights.  q8_0 bytes
//     are the A operands as stored.
//   B (activations): an f32 row x is scaled by 2^s per chunk of K so its
//     largest magnitude lies in [2^26, 2^27), rounded to the integer X and
//     split into four base-128 digits X = d0 + 2^7 d1 + 2^14 d2 + 2^21 d3
//     (d0..d2 in [0, 127], d3 signed), one B column per digit.  With one
//     token the 8 columns are (block parity, digit); with 2 or 4 tokens
//     each block parity and each pair of tokens gets its own instruction
//     (the other parity's half of K multiplies zeros) and the columns are
//     (token, digit).
//   C starts at the bit pattern of 1.5 * 2^23: every per-block column sum
//   |S| < 2^19, so the s32 result read as f32 is exactly 1.5 * 2^23 + S and
//   one FADD recovers S without an integer->float conversion.  S times the
//   block's fp16 scale is accumulated in f32 per (row, column); the digit
//   columns are recombined (x 2^(7 digit)) and scaled back by 2^-s when a
//   tile is done.  The only rounding against an f32 dot product is that of
//   x to 27 bits relative to its chunk maximum.
//
// Work split: K is cut into chunks of up to 8192 / TT elements (TT = 1, 2 or
// 4 token columns) whose activation digits fill a 33 KB shared-memory table;
// a chunk of a 16-row tile into sub-chunks of up to 32 (q4) / 16 (q8) block
// pairs, one ring stage each.  Every CTA works on one chunk (one digit table,
// built once) and streams a contiguous run of its (tile, sub-chunk) units, so
// a tile's chunk is usually summed inside one CTA.  A producer warp streams
// each unit's records (one contiguous bulk copy) into the ring with a decoded
// descriptor of the unit (full / empty mbarriers; a stage is handed back as
// soon as the consumers hold its operands in registers); eight consumer warps
// split every unit's pairs, accumulate a tile's chunk in registers and hand
// the per-warp row sums to an epilogue warp through mbarrier-guarded buffers.
// The epilogue warp sums the eight warps in fixed order; a tile whose chunk is
// whole in this CTA and the only chunk is final at once (fused epilogue:
// store / residual add / SwiGLU / RoPE + KV append); other pieces go to a
// workspace, arrivals are counted per tile with release-atomics (batched over
// four pieces), and the arrival that completes a tile sums its pieces in
// (chunk, part) order -- deterministic -- and runs the fused epilogue.
#include <cfloat>
#include <type_traits>

#include "tn_kernels.cuh"
#include "tn_ptx.cuh"

namespace tn {

// d += A B for one m16n8k32 s8 tile (A row-major 16 x 32, B column-major 32 x 8)
__device__ __forceinline__ void mma_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// 2^n as an exact float, |n| <= 126
__device__ __forceinline__ float exp2i(int n) { return __int_as_float((n + 127) << 23); }

constexpr int MMV_NW = 8;                              // consumer warps
constexpr int MMV_NE = 1;                              // epilogue warps
constexpr int MMV_UB = 4;                              // pieces per epilogue batch
constexpr int MMV_NB = MMV_NE * MMV_UB;                // partial-sum buffers
constexpr int MMV_THREADS = (MMV_NW + MMV_NE + 1) * 32;  // + one producer warp
constexpr int MMV_MAX_STAGES = 12;
constexpr int MMV_MAX_SMEM = 200 * 1024;
constexpr int MMV_CE = 8192;                           // activation elements (x tokens) per K chunk
constexpr int kMagic = 0x4B400000;                     // bits of 1.5 * 2^23
constexpr float kMagicF = 12582912.0f;
// most block pairs per sub-chunk (one ring stage), at most a chunk
__host__ __device__ constexpr int mmv_sc(int kind, int tt) {
  return (kind == MK_Q4 ? 32 : 16) < MMV_CE / tt / 64 ? (kind == MK_Q4 ? 32 : 16) : MMV_CE / tt / 64;
}

struct MmvArgs {
  const uint8_t* data;
  int rows, tiles, pairs, cols, T;
  const float* x;
  int ldx;
  float* y;
  int ldy, mode;
  int ks, ckp, nsc, scp, stages;
  uint32_t stage_bytes;
  int* err;
  int* cnt;
  float* ws;
  MvFuse f;
};

// final value v of (row, token tt); partner = value of row ^ 1 of the same token
__device__ __forceinline__ void mmv_store(const MmvArgs& a, int row, int tt, float v, float partner) {
  if (a.mode == EPI_STORE) {
    a.y[(size_t)tt * a.ldy + row] = v;
  } else if (a.mode == EPI_RESID) {
    float* py = a.y + (size_t)tt * a.ldy + row;
    *py = *py + v;
  } else if (a.mode == EPI_SWIGLU) {
    // rows (2i, 2i + 1) = (gate_i, up_i), web/inference-worker.js:567-577
    if (!(row & 1)) a.y[(size_t)tt * a.ldy + (row >> 1)] = (v / (1.0f + expf(-v))) * partner;
  } else {  // EPI_QKV_ROPE (web/inference-worker.js:528-540 and the KV push of :554)
    const MvFuse& f = a.f;
    const RowInfo ri = f.rinfo[tt];
    if (row < f.q_dim + f.kv_dim) {
      if (row & 1) return;  // handled with its even partner
      const bool isq = row < f.q_dim;
      const int rr = isq ? row : row - f.q_dim, head = rr / f.hd, i = (rr % f.hd) >> 1, half = f.hd >> 1;
      const double2 c = f.cs[(size_t)tt * half + i];
      const double av = v, bv = partner;
      const float o0 = (float)__dsub_rn(__dmul_rn(av, c.x), __dmul_rn(bv, c.y));
      const float o1 = (float)__dadd_rn(__dmul_rn(av, c.y), __dmul_rn(bv, c.x));
      if (isq) {
        float* dst = f.q_out + (size_t)tt * f.q_dim + head * f.hd;
        dst[i] = o0;
        dst[half + i] = o1;
      } else {
        const size_t ko = kv_row_off(f.kv, ri.slot, head, ri.kv_idx, f.hd);
        kv_store(f.kc, ko + i, f.kv_type, o0);
        kv_store(f.kc, ko + half + i, f.kv_type, o1);
      }
    } else {
      const int dv = row - f.q_dim - f.kv_dim;
      kv_store(f.vc, kv_row_off(f.kv, ri.slot, dv / f.hd, ri.kv_idx, f.hd) + dv % f.hd, f.kv_type, v);
    }
  }
}

// Work partition.  CTA b works on K chunk b % ks only (one digit table per
// CTA); the gk CTAs of a chunk split its units u = t * nsc + sc (tile t,
// sub-chunk sc): units [0, pool0) in contiguous runs of pool0 / gk units
// (rounded, at least nsc each, so a (tile, chunk) is split into at most two
// pieces: part 0 from sub-chunk 0, part 1 from a later one), and on chunks of
// at least 2 tiles per CTA a pool of whole tiles [pool0, NSU) (all but one
// tile per CTA below 8 tiles per CTA, else the last quarter) that the chunk's
// CTAs take in ticket order after their runs -- whole tiles, so the pool adds
// no cross-CTA pieces -- so that CTAs that got their SM slot late (and start
// with an empty ring) take fewer of them (decode bench: 93.8 -> 96.8 tok/s
// when the smaller matrices got their pool too).
__host__ __device__ __forceinline__ int mmv_chunk_ctas(int grid, int ks, int kc) { return (grid - kc + ks - 1) / ks; }
__host__ __device__ __forceinline__ int mmv_pool0(int nsu, int gk, int nsc) {
  const int q = nsu / gk;
  if (q < 2 * nsc) return nsu;
  // at least two tiles per CTA: one static tile each below 8, else the first
  // three quarters static; the rest is the pool
  const int p = q < 8 * nsc ? gk * nsc : (gk * (q - q / 4) + nsc - 1) / nsc * nsc;  // a tile boundary
  return p < nsu ? p : nsu;
}
// bytes of the per-warp row-sum buffers at the start of dynamic shared memory
__host__ __device__ constexpr int mmv_red_bytes(int tt) { return (MMV_NB * MMV_NW * 16 * tt * 4 + 127) / 128 * 128; }
constexpr int kPieceEnd = 1 << 16;  // unit descriptor flag (with the sub-chunk): the last unit of a piece

template <int KIND, int TT>
__global__ void __launch_bounds__(MMV_THREADS, 2) k_mmv(const MmvArgs a) {
  constexpr int AB = tile_a_bytes(KIND), REC = tile_rec_bytes(KIND);
  constexpr int SC = mmv_sc(KIND, TT), PPW = SC / MMV_NW, NV = 16 * TT, NC = MMV_NW * 32;
  // B column groups of 8 columns (tokens 2 cg, 2 cg + 1 x 4 digits; one token:
  // 2 block parities x 4 digits), and 32-value groups of a tile's row sums
  // (the epilogue lanes; also the workspace stride of a part)
  constexpr int NG = TT == 1 ? 1 : TT / 2;
  static_assert(TT == 1 || TT == 2 || TT == 4, "1, 2 or 4 token columns");
  constexpr int CP = MMV_CE / TT / 64;     // most pairs per chunk
  constexpr int DS = CP * 16 + 8;          // words per digit plane (skewed against bank conflicts)
  constexpr int ZERO = TT * 4 * DS;        // two zero words after the planes
  constexpr unsigned FULL = 0xffffffffu;
  // dynamic shared memory: the per-warp row sums, then the ring
  extern __shared__ __align__(128) uint8_t dyn_smem[];
  float(*red)[MMV_NW][NV] = reinterpret_cast<float(*)[MMV_NW][NV]>(dyn_smem);  // [MMV_NB][MMV_NW][NV]
  uint8_t* const ring = dyn_smem + mmv_red_bytes(TT);
  // digit planes of the current chunk: word ((tt*4 + digit)*DS + ((p*2 + q)*4 + c)*2 + h)
  // holds that digit of elements 16h + 4c .. 16h + 4c + 3 of block 2p + q
  __shared__ __align__(16) uint32_t planes[TT * 4 * DS + 2];
  __shared__ __align__(8) uint64_t full[MMV_MAX_STAGES];
  __shared__ __align__(8) uint64_t empty[MMV_MAX_STAGES];
  __shared__ __align__(8) uint64_t red_full[MMV_NB];
  __shared__ __align__(8) uint64_t red_empty[MMV_NB];
  __shared__ __align__(8) uint64_t ss_bar;  // the consumers' sums of squares are in sred
  __shared__ int last_unit[MMV_MAX_STAGES];
  __shared__ int4 udesc[MMV_MAX_STAGES];  // unit in each stage: tile (-1: no more), sub-chunk | kPieceEnd, first pair, pairs
  __shared__ int rmeta[MMV_NB][3];       // piece in each buffer: tile (-1: no more), first sub-chunk, units
  __shared__ double sred[MMV_NW][TT];
  __shared__ volatile int abort_flag;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int NSU = a.tiles * a.nsc;  // units per chunk
  const int kc0 = blockIdx.x % a.ks, gk = mmv_chunk_ctas(gridDim.x, a.ks, kc0);
  const int jc = blockIdx.x / a.ks, pool0 = mmv_pool0(NSU, gk, a.nsc);
  const int s_begin = (int)((int64_t)pool0 * jc / gk), s_end = (int)((int64_t)pool0 * (jc + 1) / gk);
  const int np0 = min(a.ckp, a.pairs - kc0 * a.ckp);  // pairs of the chunk

  if (tid == 0) {
    abort_flag = 0;
    planes[ZERO] = 0u;
    planes[ZERO + 1] = 0u;
    for (int s = 0; s < a.stages; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], MMV_NW);
      last_unit[s] = -1;
    }
    for (int b = 0; b < MMV_NB; b++) {
      mbar_init(&red_full[b], MMV_NW);
      mbar_init(&red_empty[b], 1);
    }
    mbar_init(&ss_bar, MMV_NW);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == MMV_NW + MMV_NE) {
    // ======================= producer: one bulk copy per unit into the ring
    // (weights do not depend on the previous kernel: the static run goes out
    // before any wait for it), then a descriptor without a unit
    if (lane == 0) {
      int k = 0;
      // the ring stage for unit k, once every consumer warp has read its last unit
      auto take = [&]() -> int {
        const int st = k % a.stages;
        if (k >= a.stages) {
          if (!mbar_wait_fast(&empty[st], ((k / a.stages) - 1) & 1, &abort_flag)) return -1;
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        }
        return abort_flag ? -1 : st;
      };
      auto put = [&](int st, int u, bool piece_end) {
        const int t = u / a.nsc, sc = u - t * a.nsc, first = sc * a.scp, n = max(0, min(a.scp, np0 - first));
        const uint32_t bytes = (uint32_t)n * REC;
        udesc[st] = make_int4(t, sc | (piece_end || sc == a.nsc - 1 ? kPieceEnd : 0), first, n);
        last_unit[st] = k;
        mbar_expect_tx(&full[st], bytes);  // an empty sub-chunk completes on this arrival alone
        if (bytes)
          bulk_g2s(ring + (size_t)st * a.stage_bytes,
                   a.data + ((size_t)t * a.pairs + (size_t)kc0 * a.ckp + first) * REC, bytes, &full[st]);
        k++;
      };
      auto no_more = [&](int st) {
        udesc[st] = make_int4(-1, 0, 0, 0);
        mbar_expect_tx(&full[st], 0);
      };
      bool live = true;
      for (int u = s_begin; u < s_end && live; u++) {
        const int st = take();
        if (st < 0) live = false;
        else put(st, u, u == s_end - 1);
      }
      if (pool0 < NSU) {
        // the tickets were reset by the previous launch on this matrix, which
        // may be the predecessor
        pdl_wait();
        const int ntiles = (NSU - pool0) / a.nsc;
        while (live) {
          const int r = atomicAdd(a.cnt + a.tiles + kc0, 1);  // in flight while a stage frees up
          int st = take();
          if (st < 0) break;
          if (r >= ntiles) {
            no_more(st);
            break;
          }
          for (int u = pool0 + r * a.nsc, ue = u + a.nsc; u < ue; u++) {
            if (u > pool0 + r * a.nsc && (st = take()) < 0) {
              live = false;
              break;
            }
            put(st, u, u == ue - 1);
          }
        }
        // the last CTA of the chunk past its last ticket makes the tickets
        // ready for the next launch
        __threadfence();
        if (atomicAdd(a.cnt + a.tiles + a.ks + kc0, 1) == gk - 1) {
          a.cnt[a.tiles + kc0] = 0;
          a.cnt[a.tiles + a.ks + kc0] = 0;
        }
      } else if (live) {
        const int st = take();
        if (st >= 0) no_more(st);
      }
    }
  } else if (warp < MMV_NW) {
    // ======================= consumers
    const int g = lane >> 2, c = lane & 3;
    // Activation digits are built by each warp for exactly the block pairs it
    // multiplies -- pairs sc * scp + 8 j + warp of the chunk -- with its own
    // power-of-two scale, so no CTA-wide step stands between the predecessor
    // kernel's output and the first MMA.  A lane covers one float4 of a pair:
    // elements 4 l .. 4 l + 3 (l = lane & 15), i.e. block 2p + (l >> 3),
    // elements 4 (l & 7) .., whose digits go to word 16 p + wl of each plane.
    constexpr int WP = CP / MMV_NW;  // most pairs of a chunk per warp
    constexpr int IT = WP / 2;       // two pairs per step
    const int l16 = lane & 15;
    const int wl = (l16 >> 3) * 8 + (l16 & 3) * 2 + ((l16 >> 2) & 1);
    // pair of step it of chunk kc and whether this warp multiplies it
    auto pair_of = [&](int kc, int it, bool& ok) {
      const int i = 2 * it + (lane >> 4), sc = i / PPW, jj = i - sc * PPW;
      const int pc = sc * a.scp + 8 * jj + warp;
      ok = 8 * jj + warp < a.scp && pc < min(a.ckp, a.pairs - kc * a.ckp);
      return pc;
    };
    // The RMSNorm weights of a chunk (static: no wait for the predecessor) are
    // parked in the words of digit planes 0..3 that this lane later fills with
    // its own digits, so only this lane reads them back.
    auto stage_w = [&](int kc) {
#pragma unroll
      for (int it = 0; it < IT; it++) {
        bool ok;
        const int pc = pair_of(kc, it, ok), col = kc * a.ckp * 64 + pc * 64 + l16 * 4;
        if (!ok) continue;
        float4 w4 = make_float4(0.f, 0.f, 0.f, 0.f);
        if (col < a.cols) {
          if ((reinterpret_cast<uintptr_t>(a.f.norm_w) & 15) == 0) {
            w4 = *reinterpret_cast<const float4*>(a.f.norm_w + col);
          } else {
            w4.x = a.f.norm_w[col];
            w4.y = a.f.norm_w[col + 1];
            w4.z = a.f.norm_w[col + 2];
            w4.w = a.f.norm_w[col + 3];
          }
        }
        float* pw = reinterpret_cast<float*>(planes) + pc * 16 + wl;
        pw[0] = w4.x;
        pw[DS] = w4.y;
        pw[2 * DS] = w4.z;
        pw[3 * DS] = w4.w;
      }
    };
    if (a.f.norm_w != nullptr) stage_w(kc0);
    pdl_wait();  // x is produced by the predecessor kernel
    const float* xrow[TT];
    bool xvec = true;
#pragma unroll
    for (int tt = 0; tt < TT; tt++) {
      xrow[tt] = a.x + (size_t)(tt < a.T ? (a.f.rowsel ? a.f.rowsel[tt] : tt) : 0) * a.ldx;
      xvec = xvec && (reinterpret_cast<uintptr_t>(xrow[tt]) & 15) == 0;
    }

    // RMSNorm (web/inference-worker.js:516-522) is applied to the row sums:
    // y = inv * W (x o w), inv = 1 / sqrt(mean(x^2) + 1e-5), computed by the
    // epilogue warp from the consumers' sums of squares.  With one chunk the
    // warps' digit passes below cover the row and provide those sums; with
    // several, a first pass over the row does.
    const bool ss_in_setup = a.f.norm_w != nullptr && a.ks == 1;
    if (a.f.norm_w != nullptr && a.ks > 1) {
#pragma unroll
      for (int tt = 0; tt < TT; tt++) {
        double ss = 0.0;
        if (tt < a.T)
          for (int i = tid; i < a.cols; i += NC) {
            const double v = xrow[tt][i];
            ss = fma(v, v, ss);
          }
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(FULL, ss, o);
        if (lane == 0) sred[warp][tt] = ss;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&ss_bar);
    }

    float fa[TT], fb[TT];
    auto setup = [&](int kc) {
      const int e0 = kc * a.ckp * 64;
      float v[TT][IT][4];
      // every x load is issued before any is used, so they are all in flight at once
#pragma unroll
      for (int it = 0; it < IT; it++) {
        bool ok;
        const int pc = pair_of(kc, it, ok), col = e0 + pc * 64 + l16 * 4;
        const bool valid = ok && col < a.cols;  // col % 4 == 0 and cols % 32 == 0
#pragma unroll
        for (int tt = 0; tt < TT; tt++) {
          float4 xv = make_float4(0.f, 0.f, 0.f, 0.f);
          if (valid && tt < a.T) {
            if (xvec) {
              xv = *reinterpret_cast<const float4*>(xrow[tt] + col);
            } else {
              xv.x = xrow[tt][col];
              xv.y = xrow[tt][col + 1];
              xv.z = xrow[tt][col + 2];
              xv.w = xrow[tt][col + 3];
            }
          }
          v[tt][it][0] = xv.x;
          v[tt][it][1] = xv.y;
          v[tt][it][2] = xv.z;
          v[tt][it][3] = xv.w;
        }
      }
      if (a.f.norm_w) {
        if (ss_in_setup) {
#pragma unroll
          for (int tt = 0; tt < TT; tt++) {
            double ss = 0.0;
#pragma unroll
            for (int it = 0; it < IT; it++) {
              float s4 = 0.f;  // four squares in f32, then one double add
#pragma unroll
              for (int m = 0; m < 4; m++) s4 = fmaf(v[tt][it][m], v[tt][it][m], s4);
              ss += (double)s4;
            }
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(FULL, ss, o);
            if (lane == 0) sred[warp][tt] = ss;
          }
        }
        // the parked weights, read back before this lane writes any digit
#pragma unroll
        for (int it = 0; it < IT; it++) {
          bool ok;
          const float* pw = reinterpret_cast<const float*>(planes) + pair_of(kc, it, ok) * 16 + wl;
          if (!ok) continue;
#pragma unroll
          for (int m = 0; m < 4; m++) {
            const float wv = pw[m * DS];
#pragma unroll
            for (int tt = 0; tt < TT; tt++) v[tt][it][m] *= wv;
          }
        }
      }
#pragma unroll
      for (int tt = 0; tt < TT; tt++) {
        // largest magnitude: on the bit patterns of |v|, where every NaN and
        // infinity lies at or above that of +inf
        uint32_t mb = 0u;
#pragma unroll
        for (int it = 0; it < IT; it++)
#pragma unroll
          for (int m = 0; m < 4; m++) mb = max(mb, __float_as_uint(v[tt][it][m]) & 0x7fffffffu);
        for (int o = 16; o > 0; o >>= 1) mb = max(mb, __shfl_xor_sync(FULL, mb, o));
        const bool bad = mb >= 0x7f800000u;
        const int sh = (!bad && mb != 0u) ? 26 - ilogbf(__uint_as_float(mb)) : 0;
        const int sa = sh >> 1, sb = sh - sa;
        const float pa = exp2i(sa), pb = exp2i(sb);
        fa[tt] = bad ? __int_as_float(0x7fc00000) : exp2i(-sa) * (KIND == MK_Q4 ? 0.0625f : 1.f);
        fb[tt] = exp2i(-sb);
#pragma unroll
        for (int it = 0; it < IT; it++) {
          bool ok;
          const int pc = pair_of(kc, it, ok);
          if (!ok) continue;
          // X = d0 + 2^7 d1 + 2^14 d2 + 2^21 d3 -> bytes (d0, d1, d2, d3) of one
          // word: each step doubles the bits above a digit, opening a zero bit
          // at 7, 15, 23 (u + (u & ~m) = (u & m) + 2 (u - (u & m)), modulo 2^32)
          uint32_t dw[4];
#pragma unroll
          for (int m = 0; m < 4; m++) {
            uint32_t u = (uint32_t)__float2int_rn((v[tt][it][m] * pa) * pb);
            u += u & ~0x7fu;
            u += u & ~0x7fffu;
            u += u & ~0x7fffffu;
            dw[m] = u;
          }
          // 4 x 4 byte transpose: plane d gets byte d of the four elements
          const uint32_t t0 = __byte_perm(dw[0], dw[1], 0x5140), t1 = __byte_perm(dw[0], dw[1], 0x7362);
          const uint32_t t2 = __byte_perm(dw[2], dw[3], 0x5140), t3 = __byte_perm(dw[2], dw[3], 0x7362);
          uint32_t* pw = planes + tt * 4 * DS + pc * 16 + wl;
          pw[0] = __byte_perm(t0, t2, 0x5410);
          pw[DS] = __byte_perm(t0, t2, 0x7632);
          pw[2 * DS] = __byte_perm(t1, t3, 0x5410);
          pw[3 * DS] = __byte_perm(t1, t3, 0x7632);
        }
      }
      __syncwarp();
      if (ss_in_setup && kc == 0 && lane == 0) mbar_arrive(&ss_bar);  // the row's sums of squares are out
    };

    // this lane's B columns: one token: g = (block parity sel, digit dg), the
    // other parity's half of B read from the zero words; two or more tokens:
    // column group cg of g = (token 2 cg + sel, digit dg), one instruction per
    // block parity and column group
    const int sel = g >> 2, dg = g & 3;
    int boff[2], binc[2];
    if (TT == 1) {
      boff[0] = sel == 0 ? dg * DS + c * 2 : ZERO;
      binc[0] = sel == 0 ? 16 : 0;
      boff[1] = sel == 1 ? dg * DS + 8 + c * 2 : ZERO;
      binc[1] = sel == 1 ? 16 : 0;
    } else {
      boff[0] = (sel * 4 + dg) * DS + c * 2;
      boff[1] = boff[0] + 8;
      binc[0] = binc[1] = 16;
    }
    // weights of the digit columns this lane accumulates: 2^(7 digit)
    const float wlo = (c & 1) ? 16384.f : 1.f, whi = (c & 1) ? 2097152.f : 128.f;
    setup(kc0);  // the only chunk this CTA works on
    int pi = 0, sc0 = -1;
    float acc[NG][4];
#pragma unroll
    for (int cg = 0; cg < NG; cg++) acc[cg][0] = acc[cg][1] = acc[cg][2] = acc[cg][3] = 0.f;
    // ring stage st of the current unit and the parity of its fill
    for (int st = 0, ph = 0;; (++st == a.stages) ? (st = 0, ph ^= 1) : 0) {
      if (!__all_sync(FULL, mbar_wait_fast(&full[st], ph, &abort_flag))) break;
      const int4 d = udesc[st];
      if (d.x < 0) break;
      const int t = d.x, sc = d.y & (kPieceEnd - 1), first = d.z, n = d.w;
      if (sc0 < 0) sc0 = sc;
      const uint8_t* sbase = ring + (size_t)st * a.stage_bytes;
      {
        // all pairs' operands first, so their load -> MMA -> FMA chains overlap.
        // This warp's pairs are slots j * NW + warp of the stage; slots past the
        // sub-chunk's n pairs are skipped (n is the same for the whole warp).
        constexpr int WV = AB / 512;  // 16-byte words per lane per pair
        constexpr int NQ = TT == 1 ? 1 : 2;
        uint4 wv[PPW][WV];
        uint32_t sw[PPW][NQ];  // one token: this lane's block parity; else both
        uint2 bq[PPW][2];      // up to two tokens: the B words, read here
        int pcs[PPW];          // more tokens: the pair, B read at the instruction
        const uint8_t* wbase = sbase + (size_t)warp * REC;
#pragma unroll
        for (int j = 0; j < PPW; j++) {
          if (n < SC && j * MMV_NW + warp >= n) break;
          const uint8_t* rec = wbase + j * MMV_NW * REC;
          const int pc = min(first + j * MMV_NW + warp, CP - 1);  // chunk-local pair
          pcs[j] = pc;
#pragma unroll
          for (int v = 0; v < WV; v++) wv[j][v] = *reinterpret_cast<const uint4*>(rec + lane * 16 * WV + 16 * v);
          if (TT == 1) {
            sw[j][0] = *reinterpret_cast<const uint32_t*>(rec + AB + (2 * g + (c >> 1)) * 4);
          } else {
            const uint2 s2 = *reinterpret_cast<const uint2*>(rec + AB + 8 * g);
            sw[j][0] = s2.x;
            sw[j][NQ - 1] = s2.y;
          }
          if (TT <= 2) {
#pragma unroll
            for (int q = 0; q < 2; q++) bq[j][q] = *reinterpret_cast<const uint2*>(&planes[boff[q] + pc * binc[q]]);
          }
        }
        // the operands are in registers: hand the stage back to the producer
        // now, so the ring refills while this warp computes
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
        auto compute = [&](auto all_valid) {
#pragma unroll
          for (int j = 0; j < PPW; j++) {
            if (!decltype(all_valid)::value && j * MMV_NW + warp >= n) break;
            uint32_t A[2][4];
            if (KIND == MK_Q4) {
              const uint32_t M4 = 0xF0F0F0F0u;
              const uint4 w = wv[j][0];
              A[0][0] = w.x & M4;
              A[0][1] = (w.x << 4) & M4;
              A[0][2] = w.y & M4;
              A[0][3] = (w.y << 4) & M4;
              A[1][0] = w.z & M4;
              A[1][1] = (w.z << 4) & M4;
              A[1][2] = w.w & M4;
              A[1][3] = (w.w << 4) & M4;
            } else {
              const uint4 w0 = wv[j][0], w1 = wv[j][WV - 1];
              A[0][0] = w0.x;
              A[0][1] = w0.y;
              A[0][2] = w0.z;
              A[0][3] = w0.w;
              A[1][0] = w1.x;
              A[1][1] = w1.y;
              A[1][2] = w1.z;
              A[1][3] = w1.w;
            }
#pragma unroll
            for (int q = 0; q < NQ; q++) {
              const uint32_t s32 = sw[j][q];
              const float2 d = __half22float2(*reinterpret_cast<const __half2*>(&s32));  // (row g, row g + 8)
#pragma unroll
              for (int cg = 0; cg < NG; cg++) {
                int D[4] = {kMagic, kMagic, kMagic, kMagic};
                if (TT == 1) {
                  mma_s8(D, A[0], bq[j][0].x, bq[j][1].x);
                  mma_s8(D, A[1], bq[j][0].y, bq[j][1].y);
                } else {
                  // block parity q alone: the other half of K multiplies zeros
                  const uint2 b = TT == 2 ? bq[j][q]
                                          : *reinterpret_cast<const uint2*>(
                                                &planes[boff[q] + cg * 8 * DS + pcs[j] * 16]);
                  mma_s8(D, A[0], q == 0 ? b.x : 0u, q == 1 ? b.x : 0u);
                  mma_s8(D, A[1], q == 0 ? b.y : 0u, q == 1 ? b.y : 0u);
                }
                acc[cg][0] = fmaf(d.x, __int_as_float(D[0]) - kMagicF, acc[cg][0]);
                acc[cg][1] = fmaf(d.x, __int_as_float(D[1]) - kMagicF, acc[cg][1]);
                acc[cg][2] = fmaf(d.y, __int_as_float(D[2]) - kMagicF, acc[cg][2]);
                acc[cg][3] = fmaf(d.y, __int_as_float(D[3]) - kMagicF, acc[cg][3]);
              }
            }
          }
        };
        if (n == SC) compute(std::true_type{});
        else compute(std::false_type{});
      }
      if (!(d.y & kPieceEnd)) continue;  // the piece goes on
      // end of a piece: recombine the digit columns, sum the lanes of a row,
      // undo the 2^s scaling, hand the 16 (x TT) row sums to the epilogue
      float vg[NG], vh[NG];
#pragma unroll
      for (int cg = 0; cg < NG; cg++) {
        vg[cg] = fmaf(acc[cg][1], whi, acc[cg][0] * wlo);
        vh[cg] = fmaf(acc[cg][3], whi, acc[cg][2] * wlo);
        vg[cg] += __shfl_xor_sync(FULL, vg[cg], 1);
        vh[cg] += __shfl_xor_sync(FULL, vh[cg], 1);
        if (TT == 1) {
          vg[cg] += __shfl_xor_sync(FULL, vg[cg], 2);
          vh[cg] += __shfl_xor_sync(FULL, vh[cg], 2);
        }
        // token 2 cg + (c >> 1) of the group
        constexpr int T1 = TT == 1 ? 0 : 1;
        const float sa = (c >> 1) == 0 ? fa[2 * cg] : fa[2 * cg + T1];
        const float sb = (c >> 1) == 0 ? fb[2 * cg] : fb[2 * cg + T1];
        vg[cg] = (vg[cg] * sa) * sb;
        vh[cg] = (vh[cg] * sa) * sb;
      }
      const int b = pi % MMV_NB;
      if (pi >= MMV_NB) mbar_wait_fast(&red_empty[b], ((pi / MMV_NB) - 1) & 1, &abort_flag);
      if ((c & (TT == 1 ? 3 : 1)) == 0) {
#pragma unroll
        for (int cg = 0; cg < NG; cg++) {
          const int tt = TT == 1 ? 0 : 2 * cg + (c >> 1);
          red[b][warp][tt * 16 + g] = vg[cg];
          red[b][warp][tt * 16 + g + 8] = vh[cg];
        }
      }
      if (warp == 0 && lane == 0) {
        rmeta[b][0] = t;
        rmeta[b][1] = sc0;
        rmeta[b][2] = sc - sc0 + 1;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&red_full[b]);
      pi++;
      sc0 = -1;
#pragma unroll
      for (int cg = 0; cg < NG; cg++) acc[cg][0] = acc[cg][1] = acc[cg][2] = acc[cg][3] = 0.f;
    }
    // no more pieces
    {
      const int b = pi % MMV_NB;
      if (pi >= MMV_NB) mbar_wait_fast(&red_empty[b], ((pi / MMV_NB) - 1) & 1, &abort_flag);
      if (warp == 0 && lane == 0) rmeta[b][0] = -1;
      __syncwarp();
      if (lane == 0) mbar_arrive(&red_full[b]);
    }
  } else {
    // ======================= epilogue warps
    // Pieces come in the consumers' order.  A whole (tile, chunk) with one
    // chunk is final at once; other pieces go to the workspace, and their
    // arrivals (counted in units) are published in batches of MMV_UB, one
    // release-atomic per piece issued from UB lanes at once.
    static_assert(MMV_NE == 1, "one epilogue warp");
    pdl_wait();  // y, the KV cache and the step's row table belong to earlier kernels
    const int target = a.ks * a.nsc;
    // RMSNorm factor of this lane's token in each value group, from the
    // consumers' sums of squares
    double inv[NG];
#pragma unroll
    for (int q = 0; q < NG; q++) inv[q] = 1.0;
    if (a.f.norm_w) {
      if (__all_sync(FULL, mbar_wait(&ss_bar, 0, &abort_flag))) {
#pragma unroll
        for (int q = 0; q < NG; q++) {
          const int tt = min(2 * q + (lane >> 4), TT - 1);
          double tot = 0.0;
          for (int w = 0; w < MMV_NW; w++) tot += sred[w][tt];
          inv[q] = 1.0 / sqrt(tot / a.cols + 1e-5);
        }
      }
    }
    // lane l of value group q: row l & 15 of the tile, token 2 q + (l >> 4)
    auto finish = [&](int t, const float (&vv)[NG]) {
      const int rr = lane & 15, row = t * 16 + rr;
#pragma unroll
      for (int q = 0; q < NG; q++) {
        const int tt = 2 * q + (lane >> 4);
        const float v = (float)((double)vv[q] * inv[q]);
        const float partner = __shfl_xor_sync(FULL, v, 1);
        if (lane < NV && tt < a.T && row < a.rows) mmv_store(a, row, tt, v, partner);
      }
    };
    // workspace: [chunk][tile][part][NG * 32]; a chunk of one sub-chunk is
    // never split between CTAs, so it has one part
    const int np = a.nsc > 1 ? 2 : 1;
    auto wsp = [&](int kc, int t, int part) {
      return a.ws + (((size_t)kc * a.tiles + t) * np + part) * (NG * 32) + lane;
    };
    float vb[MMV_UB][NG] = {};
    int tb[MMV_UB] = {}, ub[MMV_UB] = {};
    bool fb_[MMV_UB] = {};
    int nbat = 0;
    bool bad = false;
    auto flush = [&]() {
      if (!bad) {
        // final at once: a whole (tile, chunk) of a one-chunk matrix
#pragma unroll
        for (int i = 0; i < MMV_UB; i++)
          if (i < nbat && fb_[i] && a.ks == 1) finish(tb[i], vb[i]);
        __syncwarp();  // the workspace writes before the lanes' release atomics
        int mt = tb[0], mu = ub[0];
        bool mine = nbat > 0 && !(fb_[0] && a.ks == 1);
#pragma unroll
        for (int i = 1; i < MMV_UB; i++)
          if (lane == i) {
            mt = tb[i];
            mu = ub[i];
            mine = i < nbat && !(fb_[i] && a.ks == 1);
          }
        int old = 0;
        if (lane < nbat && mine) old = atom_add_acq_rel(a.cnt + mt, mu);
        const unsigned fin = __ballot_sync(FULL, lane < nbat && mine && old + mu == target);
        __syncwarp();  // loads below come after the acquiring atomics
#pragma unroll
        for (int i = 0; i < MMV_UB; i++) {
          if (!((fin >> i) & 1u)) continue;
          const int t = tb[i];
          // the tile's partials, summed in (chunk, part) order; 8 partials
          // (x NG values) in flight at once
          constexpr int PB = 8;
          float v[NG];
#pragma unroll
          for (int q = 0; q < NG; q++) v[q] = 0.f;
          if (lane < NV) {
            const int tot = a.ks * np;
            for (int p0 = 0; p0 < tot; p0 += PB) {
              float pv[PB][NG];
#pragma unroll
              for (int j = 0; j < PB; j++) {
                const int p = p0 + j;
                const float* src = wsp(min(p, tot - 1) / np, t, min(p, tot - 1) % np);
#pragma unroll
                for (int q = 0; q < NG; q++) pv[j][q] = p < tot ? ld_relaxed(src + q * 32) : 0.f;
              }
#pragma unroll
              for (int j = 0; j < PB; j++)
#pragma unroll
                for (int q = 0; q < NG; q++) v[q] += pv[j][q];
            }
          }
          if (lane == i) a.cnt[t] = 0;  // ready for the next launch
          finish(t, v);
        }
      }
      nbat = 0;
      bad = false;
    };
    for (int pi = 0;; pi++) {
      const int b = pi % MMV_NB;
      const bool ok = __all_sync(FULL, mbar_wait_fast(&red_full[b], (pi / MMV_NB) & 1, &abort_flag));
      const int t = rmeta[b][0], sc0 = rmeta[b][1], cnt_u = rmeta[b][2];
      if (!ok || abort_flag) {
        bad = true;
        break;
      }
      if (t < 0) break;
      float v[NG];
#pragma unroll
      for (int q = 0; q < NG; q++) {
        v[q] = 0.f;
        if (lane < NV) {
#pragma unroll
          for (int w = 0; w < MMV_NW; w++) v[q] += red[b][w][q * 32 + lane];
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&red_empty[b]);
      const bool whole = sc0 == 0 && cnt_u == a.nsc;
      if (!(whole && a.ks == 1) && lane < NV) {
        float* w0 = wsp(kc0, t, sc0 == 0 ? 0 : 1);
#pragma unroll
        for (int q = 0; q < NG; q++) {
          w0[q * 32] = v[q];
          if (whole && np == 2) w0[NG * 32 + q * 32] = 0.f;  // no second part
        }
      }
#pragma unroll
      for (int i = 0; i < MMV_UB; i++)  // (register arrays: constant indexes)
        if (i == nbat) {
#pragma unroll
          for (int q = 0; q < NG; q++) vb[i][q] = v[q];
          tb[i] = t;
          ub[i] = cnt_u;
          fb_[i] = whole;
        }
      if (++nbat == MMV_UB) flush();
    }
    if (nbat) flush();
  }

  __syncthreads();
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

// ---------------------------------------------------------------- host side
// dynamic shared memory a CTA may take next to the kernel's static arrays
template <int KIND, int TT>
static int mmv_max_dyn() {
  int dev = 0, optin = 0;
  cudaGetDevice(&dev);
  cudaFuncAttributes fa{};
  if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess ||
      cudaFuncGetAttributes(&fa, k_mmv<KIND, TT>) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return std::min(MMV_MAX_SMEM, optin - (int)fa.sharedSizeBytes);
}

template <int KIND, int TT>
static int mmv_occ(int smem) {
  int o = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, k_mmv<KIND, TT>, MMV_THREADS, smem) != cudaSuccess) {
    cudaGetLastError();
    o = 0;
  }
  return o;
}

// Two CTAs per SM when they fit (more warps to overlap the MMA work), with
// the deepest ring that keeps that occupancy; a stage is free again as soon
// as its operands are in registers, so every stage is in flight.
template <int KIND, int TT>
static void mmv_pick(MmShape* sh) {
  const int stage = (int)sh->stage_bytes, max_dyn = mmv_max_dyn<KIND, TT>();
  if (cudaFuncSetAttribute(k_mmv<KIND, TT>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_dyn) != cudaSuccess)
    cudaGetLastError();
  const int rb = mmv_red_bytes(TT);
  int best_s = 2, best_o = 0;
  for (int s = std::min(MMV_MAX_STAGES, (max_dyn - rb) / stage); s >= 2; s--) {
    // (s goes down: the first depth that reaches an occupancy is the deepest one)
    const int o = std::min(mmv_occ<KIND, TT>(rb + s * stage), 2);
    if (o > best_o) {
      best_o = o;
      best_s = s;
    }
    if (o == 2) break;
  }
  if (best_o == 0) best_o = 1;
  sh->stages = best_s;
  sh->smem = rb + best_s * stage;
  sh->ctas = best_o;
}

int mm_prepare(Matrix* m) {
  TN_REQUIRE(m->kind == MK_Q4 || m->kind == MK_Q8, TN_EINVAL, "mm_prepare: kind %d", m->kind);
  int ks_max = 1;
  size_t ws = 0;
  for (int i = 0; i < 3; i++) {
    const int tt = 1 << i;
    MmShape& sh = m->mm[i];
    const int cp = MMV_CE / tt / 64, scmax = mmv_sc(m->kind, tt);
    sh.ks = (m->pairs + cp - 1) / cp;
    sh.ckp = (m->pairs + sh.ks - 1) / sh.ks;
    sh.nsc = (sh.ckp + scmax - 1) / scmax;
    sh.scp = (sh.ckp + sh.nsc - 1) / sh.nsc;
    sh.stage_bytes = (uint32_t)scmax * tile_rec_bytes(m->kind);  // room for a full sub-chunk
    ws = std::max(ws, (size_t)sh.ks * m->tiles * 2 * 32 * std::max(1, tt / 2));
    ks_max = std::max(ks_max, sh.ks);
    // (set once per matrix, outside any stream capture)
    if (m->kind == MK_Q4) {
      if (tt == 1) mmv_pick<MK_Q4, 1>(&sh);
      else if (tt == 2) mmv_pick<MK_Q4, 2>(&sh);
      else mmv_pick<MK_Q4, 4>(&sh);
    } else {
      if (tt == 1) mmv_pick<MK_Q8, 1>(&sh);
      else if (tt == 2) mmv_pick<MK_Q8, 2>(&sh);
      else mmv_pick<MK_Q8, 4>(&sh);
    }
  }
  m->ws_floats = ws;                          // two parts per (chunk, tile)
  m->cnt_ints = (size_t)m->tiles + 2 * ks_max;  // per-tile arrivals, per-chunk tickets and done counts
  return TN_OK;
}

template <int KIND, int TT>
static int launch_mmv(const Matrix& m, int T, const float* x, int ldx, float* y, int ldy, int mode,
                      const MvFuse& f, int* err, cudaStream_t s) {
  const MmShape& sh = m.mm[TT == 1 ? 0 : TT == 2 ? 1 : 2];
  // at most one CTA per (tile, chunk), at least one per chunk
  const int grid = std::max(sh.ks, std::min(m.tiles * sh.ks, sh.ctas * num_sms()));
  const MmvArgs a{m.data, m.rows, m.tiles, m.pairs, m.cols, T, x, ldx, y, ldy, mode, sh.ks, sh.ckp, sh.nsc,
                  sh.scp, sh.stages, sh.stage_bytes, err, m.cnt, m.ws, f};
  TN_CHECK_CUDA(launch_pdl(k_mmv<KIND, TT>, dim3(grid), dim3(MMV_THREADS), (size_t)sh.smem, s, a));
  return TN_OK;
}

bool matvec_dec_ok(const Matrix& m, int T) { return (m.kind == MK_Q4 || m.kind == MK_Q8) && T >= 1 && T <= 8; }

template <int KIND>
static int launch_mmv_n(const Matrix& m, int n, const float* x, int ldx, float* y, int ldy, int mode,
                        const MvFuse& f, int* err, cudaStream_t s) {
  if (n == 1) return launch_mmv<KIND, 1>(m, n, x, ldx, y, ldy, mode, f, err, s);
  if (n == 2) return launch_mmv<KIND, 2>(m, n, x, ldx, y, ldy, mode, f, err, s);
  return launch_mmv<KIND, 4>(m, n, x, ldx, y, ldy, mode, f, err, s);
}

int matvec_dec(const Matrix& m, int T, const float* x, int ldx, float* y, int ldy, int mode, const MvFuse& f,
               int* err, cudaStream_t s) {
  TN_REQUIRE(m.kind == MK_Q4 || m.kind == MK_Q8, TN_EUNSUPPORTED, "matvec_dec: matrix kind %d", m.kind);
  TN_REQUIRE(mode != EPI_SWIGLU || (m.rows & 1) == 0, TN_EINVAL, "swiglu needs paired rows");
  TN_REQUIRE(err, TN_EINVAL, "matvec_dec: error flag required");
  TN_REQUIRE(m.ws && m.cnt, TN_ESTATE, "matvec_dec: cross-CTA workspace missing");
  // up to four tokens per launch (1, 2 or 4 token columns); each launch
  // streams the whole matrix.  (Eight columns cost as much as two launches
  // of four: the per-record digit work, not the weight stream, bounds them.)
  for (int t0 = 0; t0 < T; t0 += 4) {
    const int n = std::min(4, T - t0);
    MvFuse g = f;
    const float* xj = x;
    if (f.rowsel) g.rowsel = f.rowsel + t0;
    else xj = x + (size_t)t0 * ldx;
    if (f.rinfo) g.rinfo = f.rinfo + t0;
    if (f.cs) g.cs = f.cs + (size_t)t0 * (f.hd / 2);
    if (f.q_out) g.q_out = f.q_out + (size_t)t0 * f.q_dim;
    float* yj = y + (size_t)t0 * ldy;
    const int rc = m.kind == MK_Q4 ? launch_mmv_n<MK_Q4>(m, n, xj, ldx, yj, ldy, mode, g, err, s)
                                   : launch_mmv_n<MK_Q8>(m, n, xj, ldx, yj, ldy, mode, g, err, s);
    if (rc != TN_OK) return rc;
  }
  return TN_OK;
}

}  // namespace tn
