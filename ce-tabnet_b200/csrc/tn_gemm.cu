// tn_gemm.cu -- q4_0 / q8_0 dequant-GEMM on the 5th-generation tensor cores
// (tcgen05, accumulators in tensor memory) for steps of many tokens: prefill
// positions and fused micro-batches.
//
// The matvec of web/inference-worker.js:523-527 for T tokens at once,
// Y[t][r] = sum_k W[r][k] X[t][k], as D[M = rows][N = tokens] = A B^T: A the
// dequantised weights in tensor memory, B the activations K-major fp16 in
// shared memory, D f32 in tensor memory.
//
// Exactness.  A q4_0 weight is (n - 8) d with d an fp16 scale, a q8_0 weight
// q d: a multiple of the last place of d with at most 14 (q4) / 18 (q8)
// significant bits.  It splits into two fp16 values with no error:
//   w_hi = RN_fp16((n - 8) d)            (one HMUL2)
//   w_lo = fma_fp16(n - 8, d, -w_hi)      (one HFMA2; the exact residual has
//                                          at most 3 (q4) / 7 (q8) significant
//                                          bits on the grid of d, so it is an
//                                          fp16 value and the FMA returns it)
// An activation row is scaled by a power of two so its largest magnitude lies
// in [2^14, 2^15) and split likewise, x_hi = RN_fp16(x 2^e), x_lo =
// RN_fp16(x 2^e - x_hi) (22 significant bits of x).  Three MMAs per K step
// accumulate w_hi x_hi + w_hi x_lo + w_lo x_hi; the dropped w_lo x_lo is below
// 2^-22 of each product.  The tensor core's additions into its f32
// accumulator do not round to nearest (measured: an error that grows with the
// number of accumulating MMAs, ~1e-4 of max |y| at K = 28672), so each chunk
// of GM_CHUNK slices accumulates into one of two partial TMEM buffers
// (ping-pong) and drain warps add every finished partial into a running f32
// sum in TMEM with IEEE adds, in chunk order (measured ~1e-6 of max |y|).  The
// result is scaled back by 2^-e per token in the epilogue.
//
// CTA = one 128-row M tile (8 record tiles of the matrix's fragment-ordered
// layout) x one N tile of NT <= 128 tokens x one K split, K in slices of 64
// (one block pair):
//   warp 0       raw-weight producer: one TMA tensor copy per raw stage moves
//                the records of 8 tiles x KSL slices (small bulk copies, one
//                per record, cost ~75 ns each to issue); weights do not depend
//                on the previous kernel, so the first stages stream before the
//                dependency wait
//   warp 1       TMEM allocator and MMA issuer (one elected lane): 4 K16 steps x
//                3 MMAs per slice; tcgen05.commit frees the slice's A and B
//                stages and, every GM_CHUNK slices, hands a partial to the drain
//   warps 2..9   dequant: two warps per TMEM lane quarter, one K half each; a
//                lane dequantises 32 weights of its row and stores their fp16
//                hi / lo halves into the A stage in tensor memory (tcgen05.st).
//                Keeping A out of shared memory matters: with A written to and
//                read from shared memory every slice cost ~1 us whatever the
//                token count (shared-memory bandwidth)
//   warp 10      activation producer: the slice's x_hi / x_lo tile, written
//                pre-swizzled by k_gemm_prep, in one bulk copy
//   warps 11..14 drain + epilogue (scale, store / residual add / SwiGLU).
// Matrices with too few M tiles to fill the GPU split K over KS CTAs per
// tile: each writes its partial to a workspace, and the last to arrive (a
// counter per tile) sums the partials in split order -- deterministic -- and
// runs the epilogue.
// Every wait is bounded; a CTA that gives up drains its copies and MMAs,
// frees its TMEM and raises the error flag.
#include <cudaTypedefs.h>

#include "tn_kernels.cuh"
#include "tn_ptx.cuh"

namespace tn {

constexpr int GM_BM = 128;                     // rows per CTA
constexpr int GM_RT = GM_BM / 16;              // record tiles per CTA
constexpr int GM_DQ_WARPS = 8;                 // dequant warps: 4 lane quarters x 2 K halves
constexpr int GM_DR_WARPS = 4;                 // drain / epilogue warps
constexpr int GM_WB = 2 + GM_DQ_WARPS;         // the activation producer
constexpr int GM_WD = GM_WB + 1;               // first drain warp
constexpr int GM_THREADS = (GM_WD + GM_DR_WARPS) * 32;
constexpr int GM_CHUNK = 4;                    // K slices accumulated by the tensor core before a drain
constexpr int GM_MAX_SA = 4, GM_MAX_SB = 6, GM_MAX_RAW = 12;
constexpr int GM_A_COLS = 64;                  // TMEM columns of one A stage: hi 32 | lo 32
constexpr int GM_SPLIT_TILES = 320;            // most (tile, split) partials of a split-K launch

struct GemmArgs {
  const uint8_t* data;  // fragment-ordered records of the matrix
  int rows, tiles, pairs;
  const uint8_t* xs;    // k_gemm_prep output: [n tile][pair][hi, lo][NT][64] fp16, swizzled
  const float* xscale;  // [T] 2^-e of each token row
  int T, NT, ntiles, ks;
  float* y;
  int ldy, mode;
  int sa, sb, raw_stages, ksl;  // A stages (TMEM), B stages (smem), raw stages of ksl slices
  int sps;                      // K slices per A / B stage (a step): 2 where TMEM has room, else 1
  uint32_t acc_cols, a_col0, idesc;
  uint32_t idesc2;  // (fold) N = 2 NT: w_hi times the x_hi | x_lo rows of a B stage in one MMA
  int fold;         // partial columns [0, NT) hold hi.hi + lo.hi, [NT, 2 NT) hi.lo
  float* ws;            // split-K partials [tile][split][NT][128]
  int* cnt;             // split-K arrivals per (M tile, N tile), zero between launches
  int* err;
};

// byte offset of element (n, k) of an fp16 [rows][64] K-major tile in the
// 128-byte swizzle (8-row atoms of 1024 bytes; the 16-byte chunk index of a
// row is XORed with the row index mod 8)
__host__ __device__ __forceinline__ uint32_t sw128_off(int n, int k) {
  return (uint32_t)((n >> 3) * 1024 + (n & 7) * 128 + ((((k >> 3) ^ n) & 7) << 4) + (k & 7) * 2);
}

// shared-memory matrix descriptor of a K-major, 128-byte-swizzled tile at
// `addr` (1024-byte aligned): stride between 8-row atoms 1024 bytes,
// descriptor version 1 (sm_100), layout type 2 (SWIZZLE_128B)
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t hsub2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}
__device__ __forceinline__ void sts64(uint32_t addr, uint32_t a, uint32_t b) {
  asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(addr), "r"(a), "r"(b) : "memory");
}

// Four weights of one row: bytes u0..u3 of `u` hold (value + bias) as
// unsigned 8-bit integers; 0x64XX is the fp16 1024 + XX, so subtracting
// (1024 + bias) gives the signed value exactly.  Returns hi pair (0,1), (2,3)
// and lo pair (0,1), (2,3) for the scale d (fp16, both halves).
__device__ __forceinline__ void dq4(uint32_t u, uint32_t d2, uint32_t off2, uint32_t (&hi)[2], uint32_t (&lo)[2]) {
  const uint32_t p0 = __byte_perm(u, 0x64646464u, 0x4140), p1 = __byte_perm(u, 0x64646464u, 0x4342);
  const uint32_t v0 = hsub2(p0, off2), v1 = hsub2(p1, off2);
  hi[0] = hmul2(v0, d2);
  hi[1] = hmul2(v1, d2);
  lo[0] = hfma2(v0, d2, hi[0] ^ 0x80008000u);
  lo[1] = hfma2(v1, d2, hi[1] ^ 0x80008000u);
}

// the pipeline's waits are on its critical path: no suspend-time hint
#ifndef GM_WAIT
#define GM_WAIT mbar_wait_fast
#endif

__device__ __forceinline__ void drain_bar() { asm volatile("bar.sync 1, %0;" ::"n"(GM_DR_WARPS * 32) : "memory"); }

// SPS: K slices per A / B stage (GemmArgs::sps)
template <int KIND, int SPS>
__global__ void __launch_bounds__(GM_THREADS, 1) k_gemm(const GemmArgs a, const __grid_constant__ CUtensorMap wmap) {
  constexpr int REC = tile_rec_bytes(KIND), AB = tile_a_bytes(KIND);
  extern __shared__ uint8_t gsm_dyn[];
  __shared__ __align__(8) uint64_t rfull[GM_MAX_RAW], rempty[GM_MAX_RAW];
  __shared__ __align__(8) uint64_t afull[GM_MAX_SA], aempty[GM_MAX_SA];
  __shared__ __align__(8) uint64_t bfull[GM_MAX_SB], bempty[GM_MAX_SB];
  __shared__ __align__(8) uint64_t pfull[2], pempty[2];
  __shared__ __align__(8) uint64_t accbar;
  __shared__ uint32_t tmem_base;
  __shared__ int last_raw[GM_MAX_RAW], last_b[GM_MAX_SB];
  __shared__ int split_last;
  __shared__ volatile int abort_flag;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // launch order: N tiles fastest, then K splits, then M tiles (the CTAs of
  // one M tile are neighbours and share its raw weights in L2)
  const int nt = (int)(blockIdx.x % a.ntiles);
  const int sp = (int)((blockIdx.x / a.ntiles) % a.ks), mt = (int)(blockIdx.x / a.ntiles / a.ks);
  const int t0 = mt * GM_RT;
  const int kb = (int)((int64_t)a.pairs * sp / a.ks), ke = (int)((int64_t)a.pairs * (sp + 1) / a.ks);
  const int K = ke - kb;  // slices of this split
  const uint32_t sbase = (smem_u32(gsm_dyn) + 1023u) & ~1023u;
  uint8_t* const smem = gsm_dyn + (sbase - smem_u32(gsm_dyn));
  const uint32_t bbytes = 2u * (uint32_t)a.NT * 128u;  // one slice's x_hi | x_lo tile
  const uint32_t bstage = bbytes * (uint32_t)SPS;
  uint8_t* const raw = smem + (size_t)a.sb * bstage;
  const int NG = (K + SPS - 1) / SPS;  // steps of SPS slices
  const uint32_t acols = (uint32_t)(GM_A_COLS * SPS);  // TMEM columns of an A stage
  const uint32_t raw_stage = (uint32_t)(GM_RT * a.ksl * REC);  // [8 tiles][ksl slices][record]

  if (tid == 0) {
    abort_flag = 0;
    for (int r = 0; r < a.raw_stages; r++) {
      mbar_init(&rfull[r], 1);
      mbar_init(&rempty[r], GM_DQ_WARPS);
      last_raw[r] = -1;
    }
    for (int s = 0; s < a.sa; s++) {
      // one dequant warp per lane quarter and slice, and with as many B as A
      // stages the B tile's copy too (one barrier for the MMA issuer to test)
      mbar_init(&afull[s], GM_DQ_WARPS / 2 * SPS + (a.sa == a.sb ? 1 : 0));
      mbar_init(&aempty[s], 1);
    }
    for (int s = 0; s < a.sb; s++) {
      mbar_init(&bfull[s], 1);
      mbar_init(&bempty[s], 1);
      last_b[s] = -1;
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&pfull[b], 1);
      mbar_init(&pempty[b], GM_DR_WARPS);
    }
    mbar_init(&accbar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc(&tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_launch_dependents();
  const uint32_t tmem = tmem_base;

  // The producer and MMA warps run their loops with all 32 lanes converged
  // (waits on every lane, one lane issues).
  if (warp == 0) {
    // ================= raw weights: stage q holds slices q ksl .. of the 8 record tiles
    if (lane == 0) tma_prefetch_map(&wmap);
    const int NQ = (K + a.ksl - 1) / a.ksl;
    for (int q = 0; q < NQ; q++) {
      const int r = q % a.raw_stages;
      if (q >= a.raw_stages) {
        if (!__all_sync(0xffffffffu, GM_WAIT(&rempty[r], ((q / a.raw_stages) - 1) & 1, &abort_flag))) break;
        // the dequant warps read this slot with generic loads; the refill is an
        // async-proxy write: order the two proxies
        fence_async_smem();
      }
      if (lane == 0) {
        // (the box is whole even where it reaches past the split or the last
        // tile: tiles past the matrix read as zero, extra slices go unused)
        mbar_expect_tx(&rfull[r], raw_stage);
        tma_load_3d(raw + (size_t)r * raw_stage, &wmap, 0, kb + q * a.ksl, t0, &rfull[r]);
        last_raw[r] = q;
      }
      __syncwarp();
    }
  } else if (warp == GM_WB) {
    // ================= activations: a step's x_hi | x_lo tiles (contiguous in
    // xs, slice after slice), one bulk copy
    pdl_wait();  // xs is written by the previous kernel
    for (int g = 0; g < NG; g++) {
      const int s = g % a.sb, nk = min(SPS, K - g * SPS);
      // (with as many A as B stages, one commit frees both: the A stage's barrier)
      uint64_t* const empty = a.sa == a.sb ? &aempty[s] : &bempty[s];
      if (g >= a.sb && !__all_sync(0xffffffffu, GM_WAIT(empty, ((g / a.sb) - 1) & 1, &abort_flag))) break;
      if (lane == 0) {
        uint64_t* const full = a.sa == a.sb ? &afull[s] : &bfull[s];
        mbar_expect_tx(full, bbytes * nk);
        bulk_g2s(smem + (size_t)s * bstage, a.xs + ((size_t)nt * a.pairs + kb + g * SPS) * bbytes, bbytes * nk, full);
        last_b[s] = g;
      }
      __syncwarp();
    }
  } else if (warp == 1) {
    // ================= MMA issuer
    // A barrier test costs hundreds of cycles even when the phase is already
    // complete, and the issuer's loop sets the pace at a few tokens: the next
    // slice's stages are tested before this slice's MMAs are issued (the
    // test's latency hides behind the issue) and waited for only if not ready.
    bool ready = false;
    for (int g = 0; g < NG; g++) {
      // chunk c (GM_CHUNK slices, whole steps) accumulates into partial buffer
      // c & 1 (TMEM columns (1 + b) acc_cols ..)
      const int k0 = g * SPS, nk = min(SPS, K - k0);
      const int c = k0 / GM_CHUNK, b = c & 1;
      const bool first = k0 % GM_CHUNK == 0, last = (k0 + nk) % GM_CHUNK == 0 || k0 + nk == K;
      if (first && c >= 2 && !__all_sync(0xffffffffu, GM_WAIT(&pempty[b], ((c >> 1) - 1) & 1, &abort_flag))) break;
      const int sa = g % a.sa, sb = g % a.sb;
      const bool merged = a.sa == a.sb;  // afull also counts the B copy
      if (!ready && !__all_sync(0xffffffffu, GM_WAIT(&afull[sa], (g / a.sa) & 1, &abort_flag) &&
                                                 (merged || GM_WAIT(&bfull[sb], (g / a.sb) & 1, &abort_flag))))
        break;
      tc_fence_after();
      bool next = false;
      if (g + 1 < NG) {
        const bool na = mbar_test_wait(&afull[(g + 1) % a.sa], ((g + 1) / a.sa) & 1);
        const bool nb = merged || mbar_test_wait(&bfull[(g + 1) % a.sb], ((g + 1) / a.sb) & 1);
        next = na && nb;
      }
      if (lane == 0) {
        const uint32_t d = tmem + (uint32_t)(1 + b) * a.acc_cols;
#pragma unroll
        for (int kk = 0; kk < SPS; kk++) {
          if (kk >= nk) break;
          const uint32_t ahi = tmem + a.a_col0 + (uint32_t)sa * acols + (uint32_t)kk * GM_A_COLS;
          const uint32_t alo = ahi + GM_A_COLS / 2;
          const uint32_t st = sbase + (uint32_t)sb * bstage + (uint32_t)kk * bbytes;
          const uint64_t bhi = sw128_desc(st), blo = sw128_desc(st + bbytes / 2);
#pragma unroll
          for (int j = 0; j < 4; j++) {
            // a K16 step: 8 TMEM columns of A, 32 bytes further along B's swizzled rows
            const uint64_t dj = (uint64_t)(2 * j);
            const uint32_t aj = (uint32_t)(8 * j);
            const uint32_t acc = !(first && kk == 0 && j == 0);
            if (a.fold) {
              // the lo rows of B follow its hi rows: one MMA over both
              umma_f16_ts(d, ahi + aj, bhi + dj, a.idesc2, acc);
              umma_f16_ts(d, alo + aj, bhi + dj, a.idesc, 1u);
            } else {
              umma_f16_ts(d, ahi + aj, bhi + dj, a.idesc, acc);
              umma_f16_ts(d, ahi + aj, blo + dj, a.idesc, 1u);
              umma_f16_ts(d, alo + aj, bhi + dj, a.idesc, 1u);
            }
          }
        }
        umma_commit(&aempty[sa]);  // the stages are free once these MMAs have read them
        if (a.sa != a.sb) umma_commit(&bempty[sb]);
        if (last) umma_commit(&pfull[b]);  // the chunk's partial is complete
      }
      __syncwarp();
      ready = __all_sync(0xffffffffu, next);
    }
    // completion of every MMA issued above (also after giving up, so the
    // TMEM is only freed when nothing writes it any more)
    if (lane == 0) umma_commit(&accbar);
    __syncwarp();
  } else if (warp >= GM_WD) {
    // ================= drain: TMEM lanes 32 (warp % 4) .. + 31 = rows of the M tile
    const int quarter = warp & 3;
    const uint32_t lanes = (uint32_t)(quarter * 32) << 16;
    const int rl = quarter * 32 + lane, row = mt * GM_BM + rl;  // M-tile row, matrix row
    const int NC = (K + GM_CHUNK - 1) / GM_CHUNK;
    const size_t tile = (size_t)mt * a.ntiles + nt;
    float* const wsp = a.ws + (tile * a.ks + sp) * (size_t)a.NT * GM_BM;  // this split's [NT][128] partial
    // scale, then store / residual add / SwiGLU one value of (row, token n)
    auto emit = [&](int n, float acc) {
      const bool tok = n < a.T;
      const float val = acc * (tok ? a.xscale[n] : 0.f);
      if (a.mode == EPI_SWIGLU) {
        const float up = __shfl_xor_sync(0xffffffffu, val, 1);
        if (tok && !(row & 1) && row + 1 < a.rows) a.y[(size_t)n * a.ldy + (row >> 1)] = (val / (1.0f + expf(-val))) * up;
      } else if (tok && row < a.rows) {
        float* py = a.y + (size_t)n * a.ldy + row;
        *py = a.mode == EPI_RESID ? *py + val : val;
      }
    };
    bool done = false;
    for (int c = 0; c < NC; c++) {
      const int b = c & 1;
      if (!__all_sync(0xffffffffu, GM_WAIT(&pfull[b], (c >> 1) & 1, &abort_flag))) break;
      tc_fence_after();
      const uint32_t pb = tmem + lanes + (uint32_t)(1 + b) * a.acc_cols, sbuf = tmem + lanes;
      const bool fin = c == NC - 1;
      for (int c0 = 0; c0 < a.NT; c0 += 16) {
        uint32_t v[16], u[16];
        tmem_ld16(pb + (uint32_t)c0, v);
        if (a.fold) {
          uint32_t w2[16];  // the hi.lo products
          tmem_ld16(pb + (uint32_t)(a.NT + c0), w2);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; j++) v[j] = __float_as_uint(__uint_as_float(v[j]) + __uint_as_float(w2[j]));
        }
        if (c > 0) tmem_ld16(sbuf + (uint32_t)c0, u);
        tmem_ld_wait();
        if (c > 0) {
#pragma unroll
          for (int j = 0; j < 16; j++) v[j] = __float_as_uint(__uint_as_float(u[j]) + __uint_as_float(v[j]));
        }
        if (!fin) {
          tmem_st16(sbuf + (uint32_t)c0, v);  // running sum of the chunks so far
        } else if (a.ks == 1) {
          pdl_wait();  // y belongs to earlier kernels
#pragma unroll
          for (int j = 0; j < 16; j++) emit(nt * a.NT + c0 + j, __uint_as_float(v[j]));
        } else {
#pragma unroll
          for (int j = 0; j < 16; j++) wsp[(size_t)(c0 + j) * GM_BM + rl] = __uint_as_float(v[j]);
        }
      }
      if (fin) {
        done = true;
        break;
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&pempty[b]);  // the partial buffer may be overwritten
    }
    tc_fence_before();
    if (a.ks > 1) {
      // every drain warp reaches this barrier (also after giving up)
      __threadfence();
      drain_bar();
      if (tid == GM_WD * 32) {
        int last = 0;
        if (done && !abort_flag) last = atom_add_acq_rel(a.cnt + tile, 1) == a.ks - 1;
        split_last = last;
      }
      drain_bar();
      if (split_last) {
        // the other splits' partials, in split order (deterministic)
        __threadfence();
        pdl_wait();
        for (int n0 = 0; n0 < a.NT; n0++) {
          float acc = 0.f;
          for (int q = 0; q < a.ks; q++) acc += ld_relaxed(a.ws + ((tile * a.ks + q) * a.NT + n0) * GM_BM + rl);
          emit(nt * a.NT + n0, acc);
        }
        if (tid == GM_WD * 32) a.cnt[tile] = 0;  // ready for the next launch
      }
    }
  } else {
    // ================= dequant (warps 2..9): row quarter * 32 + lane of the M
    // tile.  The two warps of a lane quarter take alternate slices (parity
    // par), each both K halves of its slice, so that two slices per quarter
    // are in flight: a slice's chain (record loads, dequant, TMEM stores and
    // their wait, the hand-off) is latency-bound.
    const int quarter = warp & 3, par = (warp - 2) >> 2;
    const uint32_t lanes = (uint32_t)(quarter * 32) << 16;
    const int m = quarter * 32 + lane;             // M-tile row
    const int tt = m >> 4, g = m & 7, u = (m >> 3) & 1;  // record tile, row g + 8 u of it
    const uint32_t off2 = KIND == MK_Q4 ? 0x64086408u : 0x64806480u;  // fp16 (1024 + bias) twice
    const int NQ = (K + a.ksl - 1) / a.ksl;
    bool live = true;
    for (int q0 = 0; q0 < NQ && live; q0++) {
      const int r = q0 % a.raw_stages, nk = min(a.ksl, K - q0 * a.ksl);
      // (a barrier wait costs hundreds of cycles even when the phase is complete:
      // one per raw stage, not one per slice)
      if (!__all_sync(0xffffffffu, GM_WAIT(&rfull[r], (q0 / a.raw_stages) & 1, &abort_flag))) break;
      if (par >= nk) {  // no slice of this stage for this warp
        __syncwarp();
        if (lane == 0) mbar_arrive(&rempty[r]);
        continue;
      }
      for (int i0 = par; i0 < nk; i0 += 2) {
        const int k = q0 * a.ksl + i0;
        // blocks 2p and 2p + 1 of this row: lane slots 4 g + c of the record
        // (c = 0..3), word 2h + kh (q4) / 4h + 2kh + u (q8) for element half h
        // of block half kh, and the row's two scales; each slot is read as
        // whole 16-byte vectors
        const uint8_t* rec = raw + (size_t)r * raw_stage + (size_t)(tt * a.ksl + i0) * REC;
        uint32_t w[2][2][4];
#pragma unroll
        for (int c = 0; c < 4; c++) {
          const uint4* slot = reinterpret_cast<const uint4*>(rec + (4 * g + c) * (AB / 32));
          if (KIND == MK_Q4) {
            const uint4 v = slot[0];  // words 0..3 = (h, kh) = (0,0) (0,1) (1,0) (1,1)
            w[0][0][c] = v.x;
            w[1][0][c] = v.y;
            w[0][1][c] = v.z;
            w[1][1][c] = v.w;
          } else {
            const uint4 v0 = slot[0], v1 = slot[1];  // words 4h + 2kh + u
            w[0][0][c] = u ? v0.y : v0.x;
            w[1][0][c] = u ? v0.w : v0.z;
            w[0][1][c] = u ? v1.y : v1.x;
            w[1][1][c] = u ? v1.w : v1.z;
          }
        }
        const uint2 sc2 = reinterpret_cast<const uint2*>(rec + AB)[g];  // scales of blocks 2p, 2p + 1
        __syncwarp();
        if (lane == 0 && i0 + 2 >= nk) mbar_arrive(&rempty[r]);  // this warp's reads of the stage are done
        const int gs = k / SPS, sa = gs % a.sa;  // this slice's step and A stage
        if (gs >= a.sa) {
          if (!__all_sync(0xffffffffu, GM_WAIT(&aempty[sa], ((gs / a.sa) - 1) & 1, &abort_flag))) {
            live = false;
            break;
          }
          tc_fence_after();
        }
#pragma unroll
        for (int kh = 0; kh < 2; kh++) {
          const uint32_t sc = kh ? sc2.y : sc2.x;
          const uint32_t d2 = __byte_perm(sc, 0, u ? 0x3232 : 0x1010);  // this row's scale, both halves
          // element e = 16 h + 4 c + i of the block = K column e of this half: fp16
          // pair (e, e + 1) goes to column e / 2
          uint32_t hi[16], lo[16];
#pragma unroll
          for (int h = 0; h < 2; h++)
#pragma unroll
            for (int c = 0; c < 4; c++) {
              uint32_t bytes;
              if (KIND == MK_Q4) {
                // byte i = (s(row g) << 4) | s(row g + 8), s = n ^ 8
                bytes = (((u == 0) ? (w[kh][h][c] >> 4) : w[kh][h][c]) & 0x0F0F0F0Fu) ^ 0x08080808u;
              } else {
                bytes = w[kh][h][c] ^ 0x80808080u;  // q8 value of row g + 8 u, biased by 128
              }
              uint32_t ph[2], pl[2];
              dq4(bytes, d2, off2, ph, pl);
              const int col = 8 * h + 2 * c;
              hi[col] = ph[0];
              hi[col + 1] = ph[1];
              lo[col] = pl[0];
              lo[col + 1] = pl[1];
            }
          const uint32_t abase =
              tmem + lanes + a.a_col0 + (uint32_t)sa * acols + (uint32_t)(k % SPS) * GM_A_COLS + (uint32_t)(16 * kh);
          tmem_st16(abase, hi);
          tmem_st16(abase + GM_A_COLS / 2, lo);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&afull[sa]);
      }
    }
    // two slices a step and an odd K: the last step has no slice of parity 1,
    // but its A stage waits for every dequant warp
    if (live && SPS == 2 && (K & 1) && par == 1) {
      const int gs = K / 2, sa = gs % a.sa;
      if (gs < a.sa || __all_sync(0xffffffffu, GM_WAIT(&aempty[sa], ((gs / a.sa) - 1) & 1, &abort_flag))) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&afull[sa]);
      }
    }
  }

  __syncthreads();
  if (tid == 0 && abort_flag) {
    // no copy may still be landing when the CTA exits
    for (int r = 0; r < a.raw_stages; r++) {
      const int q = last_raw[r];
      if (q < 0) continue;
      abort_flag = 0;
      if (!GM_WAIT(&rfull[r], (q / a.raw_stages) & 1, &abort_flag)) break;
    }
    for (int s = 0; s < a.sb; s++) {
      const int k = last_b[s];
      if (k < 0) continue;
      abort_flag = 0;
      if (!GM_WAIT(a.sa == a.sb ? &afull[s] : &bfull[s], (k / a.sb) & 1, &abort_flag)) break;
    }
    atomicExch(a.err, 1);
  }
  __syncthreads();
  if (warp == 1) {
    if (lane == 0) {
      // every MMA has completed (the commit of accbar follows the last one)
      // before the TMEM is freed, on every path
      volatile int never = 0;
      GM_WAIT(&accbar, 0, &never);
    }
    __syncwarp();  // lane 0 rejoins the MMA warp before the warp-wide dealloc
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------- prep
// One CTA per token row of the padded N range: the row's largest magnitude
// picks e (max |x| 2^e in [2^14, 2^15)); every 8-element group becomes a
// 16-byte chunk of x_hi and one of x_lo at its swizzled place in the
// (n tile, slice) tile.  Rows past T and columns past K are zero.
__global__ void __launch_bounds__(256) k_gemm_prep(const float* __restrict__ x, int ldx, const int* __restrict__ rowsel,
                                                   int T, int K, int pairs, int NT, uint8_t* __restrict__ xs,
                                                   float* __restrict__ xscale) {
  __shared__ uint32_t smax[8];
  const int n = blockIdx.x, tid = threadIdx.x;
  pdl_launch_dependents();
  pdl_wait();
  const bool valid = n < T;
  const float* row = x + (size_t)(valid ? (rowsel ? rowsel[n] : n) : 0) * ldx;
  uint32_t mb = 0u;
  if (valid)
    for (int i = tid; i < K; i += blockDim.x) mb = max(mb, __float_as_uint(row[i]) & 0x7fffffffu);
  for (int o = 16; o > 0; o >>= 1) mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, o));
  if ((tid & 31) == 0) smax[tid >> 5] = mb;
  __syncthreads();
  mb = 0u;
  for (int w = 0; w < (int)(blockDim.x >> 5); w++) mb = max(mb, smax[w]);
  // non-finite rows pass through unscaled (inf / NaN reach the output)
  int e = 0;
  if (mb != 0u && mb < 0x7f800000u) e = min(126, max(-126, 14 - ilogbf(__uint_as_float(mb))));
  const float sc = __int_as_float((e + 127) << 23);
  if (tid == 0) xscale[n] = valid ? __int_as_float((127 - e) << 23) : 0.f;
  const int ntile = n / NT, nn = n % NT;
  const size_t tile_bytes = (size_t)NT * 128;
  for (int gi = tid; gi < pairs * 8; gi += blockDim.x) {
    const int slice = gi >> 3, k = gi * 8;
    uint32_t hv[4], lv[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
      float f[2];
#pragma unroll
      for (int m = 0; m < 2; m++) {
        const int kk = k + 2 * i + m;
        f[m] = (valid && kk < K) ? row[kk] * sc : 0.f;
      }
      const __half2 h2 = __floats2half2_rn(f[0], f[1]);
      const float2 back = __half22float2(h2);
      const __half2 l2 = __floats2half2_rn(f[0] - back.x, f[1] - back.y);
      hv[i] = *reinterpret_cast<const uint32_t*>(&h2);
      lv[i] = *reinterpret_cast<const uint32_t*>(&l2);
    }
    uint8_t* base = xs + ((size_t)ntile * pairs + slice) * 2 * tile_bytes + sw128_off(nn, k & 63);
    *reinterpret_cast<uint4*>(base) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
    *reinterpret_cast<uint4*>(base + tile_bytes) = make_uint4(lv[0], lv[1], lv[2], lv[3]);
  }
}

// ---------------------------------------------------------------- host side
static int gemm_max_dyn() {
  static int v = -1;
  if (v < 0) {
    int dev = 0, optin = 0;
    cudaGetDevice(&dev);
    cudaFuncAttributes fa{};
    if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess ||
        cudaFuncGetAttributes(&fa, k_gemm<MK_Q8, 1>) != cudaSuccess) {
      cudaGetLastError();
      return 0;
    }
    v = optin - (int)fa.sharedSizeBytes;
    if (cudaFuncSetAttribute(k_gemm<MK_Q4, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, v) != cudaSuccess ||
        cudaFuncSetAttribute(k_gemm<MK_Q8, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, v) != cudaSuccess ||
        cudaFuncSetAttribute(k_gemm<MK_Q4, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, v) != cudaSuccess ||
        cudaFuncSetAttribute(k_gemm<MK_Q8, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, v) != cudaSuccess) {
      cudaGetLastError();
      v = 0;
    }
  }
  return v;
}

void gemm_tiling(int T, int* NT, int* ntiles) {
  const int nt = (T + 127) / 128;
  *ntiles = nt;
  *NT = ((((T + nt - 1) / nt) + 15) / 16) * 16;
}

// scratch layout: prepared activations | per-token scales | split-K partials
// (at most GM_SPLIT_TILES [NT][128] f32 tiles) | split-K arrival counters
struct GemmScratch {
  size_t xs, xscale, ws, cnt, total;
};
static GemmScratch gemm_layout(int T, int cols) {
  int NT, nt;
  gemm_tiling(T, &NT, &nt);
  auto al = [](size_t v) { return (v + 255) & ~(size_t)255; };
  const size_t pairs = ((size_t)cols + 63) / 64;
  GemmScratch g;
  g.xs = 0;
  g.xscale = al((size_t)nt * pairs * 2 * NT * 128);
  g.ws = g.xscale + al((size_t)nt * NT * sizeof(float));
  g.cnt = g.ws + al((size_t)GM_SPLIT_TILES * NT * GM_BM * sizeof(float));
  g.total = g.cnt + al((size_t)GM_SPLIT_TILES * sizeof(int));
  return g;
}

size_t gemm_scratch_bytes(int T, int cols) { return gemm_layout(T, cols).total; }

size_t gemm_counter_offset(int T, int cols) { return gemm_layout(T, cols).cnt; }

bool gemm_ok(const Matrix& m, int T) {
  return (m.kind == MK_Q4 || m.kind == MK_Q8) && m.has_wmap && T >= kGemmMinTokens;
}

// cuTensorMapEncodeTiled from the driver (the runtime is linked statically;
// the driver API is not linked)
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
    else
      cudaGetLastError();
  }
  return fn;
}

// The records as a 3-D tensor of 8-byte elements [tiles][pairs][REC / 8]
// (innermost first: record bytes, pair, tile); a box is one raw stage of
// 8 tiles x ksl pairs.  Global strides REC and pairs REC are multiples of 16,
// the base is a cudaMalloc pointer, the inner coordinate is always 0.
bool gemm_encode_maps(Matrix* m) {
  auto fn = encode_fn();
  if (!fn || !(m->kind == MK_Q4 || m->kind == MK_Q8)) return false;
  const cuuint64_t rec = (cuuint64_t)tile_rec_bytes(m->kind);
  const cuuint64_t dims[3] = {rec / 8, (cuuint64_t)m->pairs, (cuuint64_t)m->tiles};
  const cuuint64_t strides[2] = {rec, rec * (cuuint64_t)m->pairs};
  const cuuint32_t estr[3] = {1, 1, 1};
  for (int i = 0; i < 3; i++) {
    const cuuint32_t box[3] = {(cuuint32_t)(rec / 8), (cuuint32_t)(1 << i), (cuuint32_t)GM_RT};
    if (fn(&m->wmap[i], CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, m->data, dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return false;
  }
  return true;
}

int gemm(const Matrix& m, int T, const float* x, int ldx, const int* rowsel, float* y, int ldy, int mode,
         void* scratch, size_t scratch_bytes, int* err, cudaStream_t s) {
  TN_REQUIRE(m.kind == MK_Q4 || m.kind == MK_Q8, TN_EUNSUPPORTED, "gemm: matrix kind %d", m.kind);
  TN_REQUIRE(mode == EPI_STORE || mode == EPI_RESID || mode == EPI_SWIGLU, TN_EINVAL, "gemm: epilogue %d", mode);
  TN_REQUIRE(mode != EPI_SWIGLU || (m.rows & 1) == 0, TN_EINVAL, "swiglu needs paired rows");
  TN_REQUIRE(err, TN_EINVAL, "gemm: error flag required");
  if (T <= 0) return TN_OK;
  const size_t need = gemm_scratch_bytes(T, m.cols);
  TN_REQUIRE(scratch && scratch_bytes >= need, TN_EINVAL, "gemm: scratch of %zu bytes, %zu needed", scratch_bytes,
             need);
  TN_REQUIRE((reinterpret_cast<uintptr_t>(scratch) & 255) == 0, TN_EINVAL, "gemm: scratch must be 256-byte aligned");
  int NT, nt;
  gemm_tiling(T, &NT, &nt);
  const GemmScratch L = gemm_layout(T, m.cols);
  uint8_t* xs = (uint8_t*)scratch;
  float* xscale = (float*)(xs + L.xscale);
  TN_CHECK_CUDA(launch_pdl(k_gemm_prep, dim3(nt * NT), dim3(256), 0, s, x, ldx, rowsel, T, m.cols, m.pairs, NT, xs,
                           xscale));
  const int max_dyn = gemm_max_dyn();
  const int REC = tile_rec_bytes(m.kind);
  GemmArgs a{};
  a.data = m.data;
  a.rows = m.rows;
  a.tiles = m.tiles;
  a.pairs = m.pairs;
  a.xs = xs;
  a.xscale = xscale;
  a.T = T;
  a.NT = NT;
  a.ntiles = nt;
  a.y = y;
  a.ldy = ldy;
  a.mode = mode;
  // TMEM: running sum at column 0, partial buffers at acc_cols and 2 acc_cols,
  // then the A stages (64 columns each) in the rest of the 512 columns.  Up
  // to 32 tokens the w_hi MMA covers x_hi and x_lo at once (two MMAs per K16
  // step instead of three; the partials take 2 NT columns)
  a.fold = NT <= 32;
  a.acc_cols = (uint32_t)(((a.fold ? 2 * NT : NT) + 31) / 32 * 32);
  a.a_col0 = 3 * a.acc_cols;
  // two K slices a stage where two such stages fit (each step's barrier
  // operations then serve twice the MMAs), else one
  a.sps = (int)((512 - a.a_col0) / (2 * GM_A_COLS)) >= 2 ? 2 : 1;
  a.sa = std::min(GM_MAX_SA, (int)((512 - a.a_col0) / (GM_A_COLS * a.sps)));
  TN_REQUIRE(a.sa >= 2, TN_EUNSUPPORTED, "gemm: no room for two A stages in tensor memory");
  // shared memory: a few B stages, then as many raw stages (~18 KB boxes) as fit
  // (a copy's loaded latency is several microseconds: the ring must be deep)
  const int bb = 2 * NT * 128 * a.sps;  // a B stage
  const int mi = 2;  // boxes of 4 slices (one stage wait per 4 slices)
  a.ksl = 1 << mi;
  // as many B as A stages: one barrier per step for both (three B stages
  // next to two A stages at 128 tokens measured 1-6 % slower)
  a.sb = a.sa;
  const int raw_stage_b = GM_RT * a.ksl * REC;
  a.raw_stages = std::min(GM_MAX_RAW, (max_dyn - 1024 - a.sb * bb) / raw_stage_b);
  const int raw_bytes = a.raw_stages * raw_stage_b;
  TN_REQUIRE(a.raw_stages >= 2, TN_EUNSUPPORTED, "gemm: no room for two raw stages in shared memory");
  TN_REQUIRE(a.sb >= 2, TN_EUNSUPPORTED, "gemm: %d bytes of shared memory is too little", max_dyn);
  // kind::f16 instruction descriptor: f32 accumulator (bit 4), A and B fp16
  // (formats 0), both K-major, N >> 3 at bit 17, M >> 4 at bit 24
  a.idesc = (1u << 4) | ((uint32_t)(NT >> 3) << 17) | ((uint32_t)(GM_BM >> 4) << 24);
  a.idesc2 = (1u << 4) | ((uint32_t)((2 * NT) >> 3) << 17) | ((uint32_t)(GM_BM >> 4) << 24);
  a.err = err;
  // split K when the (M tile, N tile) grid fills at most half the SMs: at most
  // one wave, at least two accumulation chunks per split, and at most
  // GM_SPLIT_TILES partials in the workspace
  const int mtiles = (m.tiles + GM_RT - 1) / GM_RT, base = mtiles * nt, sms = num_sms();
  // (never past one wave: a CTA's start-up and drain make a second wave dearer
  // than the longer K range it saves)
  int ks = 1;
  if (2 * base <= sms) {
    ks = sms / base;
    ks = std::min(ks, std::max(1, m.pairs / (2 * GM_CHUNK)));
    ks = std::max(1, std::min(ks, GM_SPLIT_TILES / base));
  }
  a.ks = ks;
  a.ws = (float*)(xs + L.ws);
  a.cnt = (int*)(xs + L.cnt);
  const size_t smem = (size_t)a.sb * bb + raw_bytes + 1024;
  const int grid = mtiles * ks * nt;
  if (m.kind == MK_Q4)
    TN_CHECK_CUDA(launch_pdl(a.sps == 2 ? k_gemm<MK_Q4, 2> : k_gemm<MK_Q4, 1>, dim3(grid), dim3(GM_THREADS), smem, s,
                             a, m.wmap[mi]));
  else
    TN_CHECK_CUDA(launch_pdl(a.sps == 2 ? k_gemm<MK_Q8, 2> : k_gemm<MK_Q8, 1>, dim3(grid), dim3(GM_THREADS), smem, s,
                             a, m.wmap[mi]));
  return TN_OK;
}

}  // namespace tn
