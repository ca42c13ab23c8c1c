// W4A8 linear for few tokens: NVFP4 weights (E2M1 codes, E4M3 scales per 16
// along K) times MXFP8 activations (E4M3 codes, power-of-two scales per 32).
//
// The reference has no single op for this pair (linear_mx takes one block
// size); its result is aten.linear of the two operands dequantized with their
// own block sizes (src/voyager_compiler/ops/quantized.py:455-472, 522-586).
// With M <= 16 tokens the product streams the weights once and is bound by
// HBM (arithmetic intensity ~4-56 FLOP/B), so this kernel reads the packed
// weights (0.5 B + 1/16 B per weight) instead of a dequantized bf16 copy.
//
// Weights are packed once into tiles of 256 rows x 128 K, 18 KB each and
// contiguous in (row block, K chunk) order: 256 rows of 64 nibble bytes, then
// the 256 rows' 8 scale bytes.  Within a row's 64 bytes the bytes are
// permuted so that thread t of a quad finds in its 16 contiguous bytes
// exactly its mma fragment values: for each 32-block b, k = 32b + 16h +
// {2t, 2t+1, 2t+8, 2t+9} for the two MMA steps h, so every MMA covers one
// weight scale block of 16 and one token scale block of 32.
//
// The grid is persistent (one CTA per SM): CTA i takes the tiles
// [i T / G, (i + 1) T / G) of the T tiles, so every CTA streams the same
// number of bytes.  One producer warp copies its tiles with cp.async.bulk
// into an 8-deep shared-memory ring (full / empty mbarriers, bounded waits);
// 16 compute warps take 16 rows of each tile into registers, free the stage
// and run mma.sync.m16n8k16 with f16 operands:
//   weights  each nibble pair -> f16x2 (cvt.rn.f16x2.e2m1x2) times its E4M3
//            block scale (exact in f16: at most 6 significant bits in
//            [2^-10, 2688]);
//   tokens   staged once per CTA for the K chunks its tiles cover.
// A row block whose chunks all fall to one CTA is written by it (bias, bf16);
// the CTAs that share a row block add their float32 sums into a zeroed
// workspace (vector reductions, no wait), and the CTA that adds the last
// piece reads the rows back with its two epilogue warps, writes them and
// leaves the workspace zero.  One launch per call.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "vq_numerics.cuh"
#include "vq_tc.cuh"

namespace vq {
namespace w4 {

constexpr int TILE_ROWS = 256;
#ifndef VQ_W4_MT
#define VQ_W4_MT 1
#endif
constexpr int MT = VQ_W4_MT;                 // m-tiles of 16 rows per compute warp
constexpr int WROWS = 16 * MT;
constexpr int CWARPS = TILE_ROWS / WROWS;    // compute warps
constexpr int TILE_W = TILE_ROWS * 64;       // nibble bytes of a tile (128 K)
constexpr int TILE_BYTES = TILE_W + TILE_ROWS * 8;  // + scale bytes: 18432
constexpr int STAGES = 8;
constexpr int PRODUCER = CWARPS;            // warp: the bulk copies
constexpr int EPILOGUE = CWARPS + 1;        // first warp: row blocks shared with other CTAs
constexpr int EWARPS = 2;                   // epilogue warps
constexpr int THREADS = (CWARPS + 1 + EWARPS) * 32;
constexpr int TPAD = 32;   // staged token rows padded by 64 B: rows alternate bank halves
constexpr int LMAX = 19;   // K chunks of tokens a CTA stages (16 tokens: 4.25 KB each)

// wait-timeout codes (the call's error word and the sticky one)
constexpr int ERR_TIMEOUT_FULL = 21;   // a compute warp waited for a tile
constexpr int ERR_TIMEOUT_EMPTY = 22;  // the producer waited for a free stage
constexpr int ERR_TIMEOUT_DRAIN = 23;  // the producer waited for its last copies
constexpr int ERR_TIMEOUT_FLUSH = 24;  // an epilogue warp waited for the compute warps' sums
constexpr int ERR_TIMEOUT_STAGED = 25;  // the producer waited for the tokens to be staged
#ifndef VQ_W4_FILL0
#define VQ_W4_FILL0 4
#endif
constexpr int FILL0 = VQ_W4_FILL0;  // tiles in flight before the tokens are staged

struct Args {
  const uint8_t* wt;   // packed tiles [row blocks][chunks][TILE_BYTES]
  const uint16_t* ac;  // bf16 [M, K] token codes
  const uint16_t* as;  // bf16 [M, K/32] token block scales
  const uint16_t* bias;  // bf16 [N] or null
  uint16_t* out;       // bf16 [M, N]
  float* acc;          // [row blocks * 256][16 tokens]: zero on entry, left zero
  int* done;           // [row blocks] pieces added: zero on entry, left zero
  int* err;            // first wait timeout of this launch (may be null)
  int M, N, K, chunks, tiles, G;
};

__device__ __forceinline__ uint32_t e2m1x2_to_f16x2(uint32_t byte) {
  uint32_t r;
  asm("{\n\t.reg .b8 t;\n\tcvt.u8.u32 t, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, t;\n\t}" : "=r"(r) : "r"(byte));
  return r;
}
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t two_bytes) {
  uint32_t r;
  asm("{\n\t.reg .b16 t;\n\tcvt.u16.u32 t, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, t;\n\t}" : "=r"(r) : "r"(two_bytes));
  return r;
}
// The four E2M1 pairs of a word (its bytes, low first) as f16x2.
__device__ __forceinline__ void e2m1x8_to_f16x2(uint32_t w, uint32_t (&r)[4]) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\tmov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\tcvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\tcvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
      : "r"(w));
}
// The two E4M3 pairs of a word (its 16-bit halves, low first) as f16x2.
__device__ __forceinline__ void e4m3x4_to_f16x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
  asm("{\n\t.reg .b16 h0, h1;\n\tmov.b32 {h0, h1}, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, h0;\n\tcvt.rn.f16x2.e4m3x2 %1, h1;\n\t}"
      : "=r"(lo), "=r"(hi)
      : "r"(w));
}
__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  __half2 r = __hmul2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ void mma_f16(float* d, uint32_t a0, uint32_t a1, uint32_t a2,
                                        uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void red_add2(float* p, float a, float b) {
  asm volatile("red.relaxed.gpu.global.add.v2.f32 [%0], {%1, %2};" ::"l"(p), "f"(a), "f"(b)
               : "memory");
}
__device__ __forceinline__ void consumers_sync() {  // the compute warps only
  asm volatile("bar.sync 1, %0;" ::"n"(CWARPS * 32) : "memory");
}
__device__ __forceinline__ void epilogue_sync() {  // the epilogue warps only
  asm volatile("bar.sync 2, %0;" ::"n"(EWARPS * 32) : "memory");
}

// a * (b.lo, b.lo) / a * (b.hi, b.hi): the broadcast is an operand select of
// the f16x2 multiply
__device__ __forceinline__ uint32_t hmul2_lo(uint32_t a, uint32_t b) {
  __half2 r = __hmul2(*reinterpret_cast<__half2*>(&a), __low2half2(*reinterpret_cast<__half2*>(&b)));
  return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t hmul2_hi(uint32_t a, uint32_t b) {
  __half2 r = __hmul2(*reinterpret_cast<__half2*>(&a), __high2half2(*reinterpret_cast<__half2*>(&b)));
  return *reinterpret_cast<uint32_t*>(&r);
}
// programmatic dependent launch: let the next grid on the stream start, and
// wait for the grids this one depends on (their writes visible)
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Staged position of the token value at offset kk of a CTA's staged K:
// within each 32-block, thread t's B fragments of the two MMA steps h
// (k = 16h + {2t, 2t+1, 2t+8, 2t+9}) are 8 consecutive halves, one 16-byte
// load.
__device__ __forceinline__ int tok_pos(int kk) {
  const int r = kk & 31, h = r >> 4, q = r & 15;
  return (kk & ~31) + ((q & 7) >> 1) * 8 + h * 4 + (q >> 3) * 2 + (q & 1);
}

// One K chunk (128) of a warp's 32 weight rows against the staged tokens:
// wc / scc the chunk's weight bytes and scale bytes, kc its offset in the
// staged tokens, NT token halves of 8 (1: at most 8 tokens).  SCALED: the
// staged tokens already carry their block scales (relative to the token's
// largest, exact in f16) and the MMAs accumulate straight into acc;
// otherwise they are the raw E4M3 codes and each 32-block's float32 sums
// are multiplied by the token block scales in tsc.  Even and odd 32-blocks
// accumulate into acc[0] and acc[1]: two MMA chains instead of one.
template <int NT, bool SCALED>
__device__ __forceinline__ void w4a8_chunk(const uint4 (&wc)[2 * MT], const uint2 (&scc)[2 * MT], int kc,
                                           const uint16_t* tok, const float* tsc, int ks, int nkb,
                                           int g, int t, float (&acc)[2][MT][NT][4]) {
  // the rows' 8 block scales as f16 pairs (2q, 2q + 1)
  uint32_t scl[2 * MT][4];
#pragma unroll
  for (int r = 0; r < 2 * MT; ++r) {
    e4m3x4_to_f16x2(scc[r].x, scl[r][0], scl[r][1]);
    e4m3x4_to_f16x2(scc[r].y, scl[r][2], scl[r][3]);
  }
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    uint4 bt[NT];  // token g (+ 8 nt) of block b: (h0 lo, h0 hi, h1 lo, h1 hi) f16 pairs
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
      bt[nt] = *reinterpret_cast<const uint4*>(tok + (8 * nt + g) * ks + kc + 32 * b + 8 * t);
    float d[MT][NT][4];
    if constexpr (!SCALED) {
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int v = 0; v < 4; ++v) d[mt][nt][v] = 0.f;
    }
    auto& dst = *[&]() {
      if constexpr (SCALED) return &acc[b & 1];
      else return &d;
    }();
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      // this block's codes of rows g (A) and g + 8 (B) of m-tile mt: byte
      // 2h + u holds the pair of MMA step h, k 2t (+8u)
      uint32_t da[4], db[4];
      e2m1x8_to_f16x2((&wc[2 * mt].x)[b], da);
      e2m1x8_to_f16x2((&wc[2 * mt + 1].x)[b], db);
      // block scales 2b, 2b + 1 of the two rows as f16 pairs
      const uint32_t pa = scl[2 * mt][b], pb = scl[2 * mt + 1][b];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        auto mul = [h](uint32_t x, uint32_t s) { return h ? hmul2_hi(x, s) : hmul2_lo(x, s); };
        const uint32_t a0 = mul(da[2 * h], pa), a2 = mul(da[2 * h + 1], pa);
        const uint32_t a1 = mul(db[2 * h], pb), a3 = mul(db[2 * h + 1], pb);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
          mma_f16(dst[mt][nt], a0, a1, a2, a3, h ? bt[nt].z : bt[nt].x, h ? bt[nt].w : bt[nt].y);
      }
    }
    if constexpr (!SCALED) {
      // token block scales: C columns are tokens 8 nt + 2t, + 1
      const int kb = kc / 32 + b;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const float s0 = tsc[(8 * nt + 2 * t) * nkb + kb];
        const float s1 = tsc[(8 * nt + 2 * t + 1) * nkb + kb];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          float(&a)[4] = acc[b & 1][mt][nt];
          a[0] = fmaf(d[mt][nt][0], s0, a[0]);
          a[1] = fmaf(d[mt][nt][1], s1, a[1]);
          a[2] = fmaf(d[mt][nt][2], s0, a[2]);
          a[3] = fmaf(d[mt][nt][3], s1, a[3]);
        }
      }
    }
  }
}

// The CTA whose tile range holds tile x (ranges [i T / G, (i + 1) T / G)).
// 32-bit unsigned arithmetic: the launcher guarantees T * G < 2^32.
__device__ __forceinline__ int cta_of(uint32_t x, uint32_t T, uint32_t G) {
  return (int)(((x + 1) * G - 1) / T);
}
__device__ __forceinline__ int range_start(uint32_t i, uint32_t T, uint32_t G) {
  return (int)(i * T / G);
}

// A warp's rows' loop over the CTA's tiles, for one token staging (SCALED or
// not).  Flushes each row block as its last chunk in this CTA is done: the
// whole row block straight to the output; this CTA's piece of a row block
// shared with other CTAs added into the workspace, with an arrival on the
// flush barrier of its slot (0: the CTA's first row block, 1: its last) for
// the epilogue warps, and no wait.
template <int NT, bool SCALED>
__device__ __forceinline__ void consume(const Args& p, const uint8_t* ring, uint32_t full0,
                                        uint32_t empty0, int t0, int t1, int cstart,
                                        const uint16_t* tok, const float* tsc, int ks, int nkb,
                                        const float (&mul)[NT][2], uint32_t flushed0) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, g = lane >> 2, t = lane & 3;
  const int lrow = warp * WROWS + g;  // this thread's tile rows lrow + 8i, i < 2 MT
  float acc2[2][MT][NT][4] = {};
  bool ok = true;
  // the tile at ring position k: wait for it, take this thread's rows
  auto take = [&](int k, uint4 (&w)[2 * MT], uint2 (&sc)[2 * MT]) {
    const int s = k % STAGES;
    ok = ok && tc::mbar_wait_warp(full0 + 8 * s, (uint32_t)(k / STAGES) & 1u, p.err,
                                  ERR_TIMEOUT_FULL);
    if (ok) {
      const uint8_t* st = ring + (size_t)s * TILE_BYTES;
#pragma unroll
      for (int r = 0; r < 2 * MT; ++r) {
        w[r] = *reinterpret_cast<const uint4*>(st + (lrow + 8 * r) * 64 + t * 16);
        sc[r] = *reinterpret_cast<const uint2*>(st + TILE_W + (lrow + 8 * r) * 8);
      }
    }
  };
  auto release = [&](int k) {  // the stage's rows are in registers
    __syncwarp();
    if (ok && lane == 0) tc::mbar_arrive(empty0 + 8 * (k % STAGES));
  };
  // software pipeline: tile k + 1 is taken from shared memory while tile k
  // is computed, and its stage freed after
  uint4 w[2 * MT], wn[2 * MT];
  uint2 sc[2 * MT], scn[2 * MT];
  take(0, w, sc);
  release(0);
  // tile i is chunk c of row block rb, staged chunk j
  int c = cstart, j = 0, rb = t0 / p.chunks;
  for (int i = t0, k = 0; i < t1; ++i, ++k) {
    const bool more = i + 1 < t1;
    if (more) take(k + 1, wn, scn);
    if (ok) w4a8_chunk<NT, SCALED>(w, sc, j * 128, tok, tsc, ks, nkb, g, t, acc2);
    if (more) {
      release(k + 1);
#pragma unroll
      for (int r = 0; r < 2 * MT; ++r) {
        w[r] = wn[r];
        sc[r] = scn[r];
      }
    }
    if (++j == p.chunks) j = 0;
    if (++c < p.chunks && more) continue;
    // ---- flush row block rb: rows rb * 256 + lrow + 8i (+ 16 mt, + 8 for c2/c3)
    const int64_t first = (int64_t)rb * p.chunks, lastt = first + p.chunks - 1;
    float acc[MT][NT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          acc[mt][nt][v] = (acc2[0][mt][nt][v] + acc2[1][mt][nt][v]) * mul[nt][v & 1];
          acc2[0][mt][nt][v] = 0.f;
          acc2[1][mt][nt][v] = 0.f;
        }
    if (first >= t0 && lastt < t1) {
      // the whole row block: C fragment rows g / g + 8, tokens 8 nt + 2t, + 1
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const int row = rb * TILE_ROWS + lrow + 16 * mt + 8 * (v >> 1);
          if (row >= p.N) continue;
          const float bv = p.bias ? bf2f(p.bias[row]) : 0.f;
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const int tk = 8 * nt + 2 * t + (v & 1);
            if (tk < p.M) p.out[(size_t)tk * p.N + row] = (uint16_t)f2bf(acc[mt][nt][v] + bv);
          }
        }
    } else {
      // this CTA's piece of a shared row block: rows (local) lrow + 16 mt
      // + 8u, tokens 8 nt + 2t, + 1
      float* ws = p.acc + (size_t)rb * TILE_ROWS * 16;
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int u = 0; u < 2; ++u)
            red_add2(ws + (lrow + 16 * mt + 8 * u) * 16 + 8 * nt + 2 * t, acc[mt][nt][2 * u],
                     acc[mt][nt][2 * u + 1]);
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(flushed0 + 8 * (rb == t0 / p.chunks ? 0 : 1));
    }
    if (c == p.chunks) {
      c = 0;
      ++rb;
    }
  }
}

// The epilogue warps: for each row block this CTA shares with others (its
// first and / or last), once the compute warps have added their sums, the
// first epilogue warp counts the piece in; the CTA that adds the last piece
// reads the row block back with all its epilogue warps (rows below N, tokens
// below M), adds the bias, writes bf16 and leaves the workspace and the
// counter at zero.  The compute warps' additions reach the whole GPU through
// the flush barrier (release / acquire in the CTA) and the counting warp's
// device-scope fence before the counter; the decision reaches the other
// epilogue warps through shared memory and a named barrier that every
// epilogue warp reaches, whatever its own wait gave.
template <int NT>
__device__ __forceinline__ void epilogue(const Args& p, int t0, int t1, uint32_t flushed0,
                                         int* last_flag) {
  const int lane = threadIdx.x % 32, ew = threadIdx.x / 32 - EPILOGUE;
  const uint32_t T = p.tiles, G = p.G;
  const int rbs[2] = {t0 / p.chunks, (t1 - 1) / p.chunks};
  for (int slot = 0; slot < 2; ++slot) {
    const int rb = rbs[slot];
    if (slot == 1 && rb == rbs[0]) break;
    const int64_t first = (int64_t)rb * p.chunks, lastt = first + p.chunks - 1;
    if (first >= t0 && lastt < t1) continue;  // whole: written by the compute warps
    const bool ok = tc::mbar_wait_warp(flushed0 + 8 * slot, 0, p.err, ERR_TIMEOUT_FLUSH);
    if (ew == 0) {
      int is_last = 0;
      if (ok) {
        __threadfence();
        if (lane == 0) {
          const int prev = atomicAdd(p.done + rb, 1);
          is_last = prev == cta_of((uint32_t)lastt, T, G) - cta_of((uint32_t)first, T, G);
          if (is_last) p.done[rb] = 0;
        }
        is_last = __shfl_sync(0xFFFFFFFFu, is_last, 0);
      }
      if (lane == 0) last_flag[slot] = is_last;
    }
    epilogue_sync();
    if (!last_flag[slot]) continue;
    __threadfence();
    float* ws = p.acc + (size_t)rb * TILE_ROWS * 16;
    const int nrow = min(TILE_ROWS, p.N - rb * TILE_ROWS);
    const int nv = (p.M + 3) / 4;  // float4 of a row's sums
    // rows ew * 32 + lane + 32 EWARPS i, all loads first
    constexpr int RL = TILE_ROWS / (32 * EWARPS);
    float4 q[RL][2 * NT];
#pragma unroll
    for (int i = 0; i < RL; ++i) {
      const int r = ew * 32 + lane + 32 * EWARPS * i;
#pragma unroll
      for (int v = 0; v < 2 * NT; ++v)
        q[i][v] = r < nrow && v < nv ? __ldcg(reinterpret_cast<const float4*>(ws + r * 16) + v)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int i = 0; i < RL; ++i) {
      const int r = ew * 32 + lane + 32 * EWARPS * i;
      if (r >= nrow) continue;
      const int row = rb * TILE_ROWS + r;
      const float bv = p.bias ? bf2f(p.bias[row]) : 0.f;
#pragma unroll
      for (int v = 0; v < 2 * NT; ++v) {
        if (v >= nv) continue;
        reinterpret_cast<float4*>(ws + r * 16)[v] = make_float4(0.f, 0.f, 0.f, 0.f);
        const float s4[4] = {q[i][v].x, q[i][v].y, q[i][v].z, q[i][v].w};
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (4 * v + e < p.M) p.out[(size_t)(4 * v + e) * p.N + row] = (uint16_t)f2bf(s4[e] + bv);
      }
    }
  }
}

// Shared memory: the ring, then the staged tokens f16 [8 NT][L * 128 +
// TPAD] in fragment order (tok_pos), their block scales float [8 NT][4 L],
// the per-token exponents, a flag and the mbarriers (full, empty, flushed,
// staged).
__host__ __device__ constexpr int tok_offset() { return STAGES * TILE_BYTES; }
__host__ __device__ constexpr int smem_bytes(int nt, int L) {
  return STAGES * TILE_BYTES + 8 * nt * (L * 128 + TPAD) * 2 + 8 * nt * L * 4 * 4 + 16 * 4 + 16 +
         (2 * STAGES + 3) * 8 + 8;
}

// Tokens are staged once per CTA as f16 c * 2^(e - E): c the E4M3 code, 2^e
// its block scale, E the largest block-scale exponent of the token in the
// staged chunks; every such product is exact in f16 when no block scale is
// more than 2^15 below the token's largest (checked block by block), and the
// sums are multiplied by 2^E when a row block is flushed.  A CTA whose
// tokens fail the check (or carry scales that are not positive normal powers
// of two) stages the raw codes and multiplies each 32-block's float32 sums by
// the block scales instead.
template <int NT>
__global__ void __launch_bounds__(THREADS, 1) k_w4a8(const __grid_constant__ Args p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t T = p.tiles, G = p.G;
  const int t0 = range_start(blockIdx.x, T, G), t1 = range_start(blockIdx.x + 1, T, G);
  const int cstart = t0 % p.chunks, L = min(t1 - t0, p.chunks);
  const int ks = L * 128 + TPAD, nkb = L * 4;
  uint8_t* ring = smem;
  uint16_t* tok = reinterpret_cast<uint16_t*>(smem + tok_offset());
  float* tsc = reinterpret_cast<float*>(tok + 8 * NT * ks);
  int* emax = reinterpret_cast<int*>(tsc + 8 * NT * nkb);  // per token: largest biased exponent
  int* flags = emax + 16;  // [0] slow, [1..2] last piece of the shared row block of slot 0 / 1
  uint64_t* bars = reinterpret_cast<uint64_t*>(
      (reinterpret_cast<uintptr_t>(flags + 4) + 7) & ~uintptr_t(7));
  const uint32_t full0 = tc::smem_u32(bars), empty0 = full0 + 8 * STAGES,
                 flushed0 = empty0 + 8 * STAGES, staged0 = flushed0 + 16;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(full0 + 8 * s, 1);
      tc::mbar_init(empty0 + 8 * s, CWARPS);
    }
    tc::mbar_init(flushed0, CWARPS);
    tc::mbar_init(flushed0 + 8, CWARPS);
    tc::mbar_init(staged0, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (threadIdx.x < 16) emax[threadIdx.x] = 0;
  if (threadIdx.x == 16) flags[0] = 0;
  __syncthreads();
  pdl_trigger();

  if (warp == PRODUCER) {
    // ---------------- producer: the CTA's tiles, in order ----------------
    // the first tiles from one lane each, at once (the weights are
    // constant: before the wait for the previous grid); the rest of the
    // ring once the tokens are staged (their loads do not queue behind the
    // whole ring), then by lane 0 as stages free up
    const int n = t1 - t0, first_fill = min(n, FILL0);
    if (lane < first_fill) {
      tc::mbar_expect_tx(full0 + 8 * lane, TILE_BYTES);
      tc::bulk_load(tc::smem_u32(ring + (size_t)lane * TILE_BYTES),
                    p.wt + (size_t)(t0 + lane) * TILE_BYTES, TILE_BYTES, full0 + 8 * lane);
    }
    if (lane == 0) {
      int k = first_fill;  // tiles issued
      const bool go = k >= n || tc::mbar_wait(staged0, 0, p.err, ERR_TIMEOUT_STAGED);
      for (; go && k < n; ++k) {
        const int s = k % STAGES;
        if (!tc::mbar_wait(empty0 + 8 * s, ((uint32_t)(k / STAGES) & 1u) ^ 1u, p.err,
                           ERR_TIMEOUT_EMPTY))
          break;
        tc::mbar_expect_tx(full0 + 8 * s, TILE_BYTES);
        tc::bulk_load(tc::smem_u32(ring + (size_t)s * TILE_BYTES),
                      p.wt + (size_t)(t0 + k) * TILE_BYTES, TILE_BYTES, full0 + 8 * s);
      }
      // no copy may land after the CTA has gone: wait for the last ones
      for (int kk = max(0, k - STAGES); kk < k; ++kk)
        tc::mbar_wait(full0 + 8 * (kk % STAGES), (uint32_t)(kk / STAGES) & 1u, p.err,
                      ERR_TIMEOUT_DRAIN);
    }
    return;
  }
  // the packed weights are constant: only the tokens, the workspace, the
  // counters and the output wait for the grids before this one
  pdl_wait();
  if (warp >= EPILOGUE) {
    epilogue<NT>(p, t0, t1, flushed0, flags + 1);
    return;
  }

  // ---------------- compute warps: stage the tokens ----------------
  // staged chunk j is K chunk (cstart + j) % chunks; rows M .. 8 NT - 1 are
  // zero tokens with zero scales: their output columns (never written) add
  // exact zeros into the shared workspace.  Item i of the codes is row
  // i / (16 L), 8 codes at K offset 8 (i % (16 L)); every thread's code
  // loads go out first, with the scale loads, in one round trip.
  // A thread's items are i = threadIdx.x + u ISTEP, u < NITEM: it steps
  // through their (row m, remainder r = i % 16 L) pairs with no division
  // past the first (the divisor 16 L is a runtime value); items of rows
  // 8 NT and on are past the end.
  constexpr int ISTEP = CWARPS * 32;
  constexpr int NITEM = (8 * NT * LMAX * 16 + ISTEP - 1) / ISTEP;
  const int L16 = L * 16;
  const int im0 = threadIdx.x / L16, ir0 = threadIdx.x - im0 * L16;
  const int im_step = ISTEP / L16, ir_step = ISTEP - im_step * L16;
  auto next_item = [&](int& m, int& r) {
    m += im_step;
    r += ir_step;
    if (r >= L16) {
      r -= L16;
      ++m;
    }
  };
  // K of staged offset 8 r: staged chunk j = r / 16 is K chunk
  // (cstart + j) % chunks, where cstart + j < 2 chunks
  auto k_of = [&](int r) {
    int c = cstart + (r >> 4);
    if (c >= p.chunks) c -= p.chunks;
    return c * 128 + (r & 15) * 8;
  };
  uint4 cvv[NITEM];
  {
    int m = im0, r = ir0;
#pragma unroll
    for (int u = 0; u < NITEM; ++u) {
      cvv[u] = make_uint4(0, 0, 0, 0);
      if (m < p.M) cvv[u] = *reinterpret_cast<const uint4*>(p.ac + (size_t)m * p.K + k_of(r));
      next_item(m, r);
    }
  }
  int slow = 0;
  {
    // scale i = m nkb + jb of the staged blocks, stepped the same way
    int m = threadIdx.x / nkb, jb = threadIdx.x - m * nkb;
    const int m_step = ISTEP / nkb, j_step = ISTEP - m_step * nkb;
    while (m < 8 * NT) {
      int c = cstart + (jb >> 2);
      if (c >= p.chunks) c -= p.chunks;
      const int kb = c * 4 + (jb & 3);
      const uint32_t sb = m < p.M ? p.as[(size_t)m * (p.K / 32) + kb] : 0u;
      tsc[m * nkb + jb] = __uint_as_float(sb << 16);
      const uint32_t ef = (sb >> 7) & 0xFFu;
      if (sb) {
        if ((sb & 0x807Fu) || ef == 0xFFu) slow = 1;  // not a positive normal power of two
        else atomicMax(&emax[m], (int)ef);
      }
      m += m_step;
      jb += j_step;
      if (jb >= nkb) {
        jb -= nkb;
        ++m;
      }
    }
  }
  consumers_sync();
  {
    int m = im0, r = ir0;
#pragma unroll
    for (int u = 0; u < NITEM; ++u, next_item(m, r)) {
      if (m >= 8 * NT) break;
      const int kk = r * 8;
      const uint32_t sb = __float_as_uint(tsc[m * nkb + (r >> 2)]) >> 16;
      // 2^d, d = e - E <= 0: an E4M3 code's last bit is >= 2^-9, so c * 2^d
      // is exact in f16 for d >= -15 (and below 448 <= 65504)
      const int d = (int)((sb >> 7) & 0xFFu) - emax[m];
      float f = 0.f;
      if (sb) {
        if (d >= -15) f = __uint_as_float((uint32_t)(d + 127) << 23);
        else slow = 1;
      }
      const uint32_t cv[4] = {cvv[u].x, cvv[u].y, cvv[u].z, cvv[u].w};
      uint16_t* row = tok + m * ks;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        __half2 h = __floats2half2_rn(bf2f(cv[q] & 0xFFFFu) * f, bf2f(cv[q] >> 16) * f);
        *reinterpret_cast<uint32_t*>(row + tok_pos(kk + 2 * q)) = *reinterpret_cast<uint32_t*>(&h);
      }
    }
  }
  if (slow) atomicOr(&flags[0], 1);
  consumers_sync();
  slow = flags[0];
  if (slow) {  // the raw codes (exact in f16), scales applied per 32-block
    int m = im0, r = ir0;
#pragma unroll
    for (int u = 0; u < NITEM; ++u, next_item(m, r)) {
      if (m >= 8 * NT) break;
      const int kk = r * 8;
      const uint32_t cv[4] = {cvv[u].x, cvv[u].y, cvv[u].z, cvv[u].w};
      uint16_t* row = tok + m * ks;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        __half2 h = __floats2half2_rn(bf2f(cv[q] & 0xFFFFu), bf2f(cv[q] >> 16));
        *reinterpret_cast<uint32_t*>(row + tok_pos(kk + 2 * q)) = *reinterpret_cast<uint32_t*>(&h);
      }
    }
    consumers_sync();
  }
  if (threadIdx.x == 0) tc::mbar_arrive(staged0);  // the producer may fill the rest of the ring
  // C fragment columns are tokens 8 nt + 2t, + 1; the scaled sums are 2^-E
  // of the token's
  const int t = lane & 3;
  float mul[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int e = emax[8 * nt + 2 * t + u];
      mul[nt][u] = slow ? 1.f : e ? __uint_as_float((uint32_t)e << 23) : 0.f;
    }
  if (slow)
    consume<NT, false>(p, ring, full0, empty0, t0, t1, cstart, tok, tsc, ks, nkb, mul, flushed0);
  else
    consume<NT, true>(p, ring, full0, empty0, t0, t1, cstart, tok, tsc, ks, nkb, mul, flushed0);
}

// Packing --------------------------------------------------------------------
// bf16 E2M1 codes [N, K] and bf16 E4M3 scales [N, K/16] -> tiles of 256 rows
// x 128 K (rows past N zero): nibbles (even k in the low nibble; byte o =
// 16b + 4i + t of a row's 64 goes to 16t + 4b + i, the order k_w4a8 reads),
// then the scale bytes.  Counts codes / scales that are not such values.
__global__ void k_w4_pack(const uint16_t* codes, const uint16_t* scales, uint8_t* wt, int N, int K,
                          int* inexact) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // one nibble byte
  const int chunks = K / 128;
  const int64_t rows = (int64_t)(N + TILE_ROWS - 1) / TILE_ROWS * TILE_ROWS;
  if (i < rows * (K / 2)) {
    const int64_t row = i / (K / 2), o = i % (K / 2);
    uint32_t q = 0;
    if (row < N) {
      const float f0 = bf2f(codes[row * K + 2 * o]), f1 = bf2f(codes[row * K + 2 * o + 1]);
      asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\tcvt.u32.u8 %0, t;\n\t}"
          : "=r"(q) : "f"(f1), "f"(f0));
      const uint32_t back = e2m1x2_to_f16x2(q);
      const float g0 = __half2float(__ushort_as_half((unsigned short)(back & 0xFFFF)));
      const float g1 = __half2float(__ushort_as_half((unsigned short)(back >> 16)));
      const int bad = (g0 != f0) + (g1 != f1);  // -0 == +0 counts as equal
      if (bad && inexact) atomicAdd(inexact, bad);
    }
    const int c = (int)(o / 64), oo = (int)(o % 64);
    const int b = oo / 16, ii = (oo % 16) / 4, t = oo % 4;
    const int64_t tile = row / TILE_ROWS * chunks + c;
    wt[tile * TILE_BYTES + (row % TILE_ROWS) * 64 + t * 16 + 4 * b + ii] = (uint8_t)q;
  }
  if (i < rows * (K / 16)) {
    const int64_t row = i / (K / 16), o = i % (K / 16);
    uint8_t v = 0;
    if (row < N) {
      const float f = bf2f(scales[row * (K / 16) + o]);
      uint16_t b;
      asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(b) : "f"(0.f), "f"(f));
      v = (uint8_t)(b & 0xFF);
      const uint32_t back = e4m3x2_to_f16x2(v);
      const float g = __half2float(__ushort_as_half((unsigned short)(back & 0xFFFF)));
      if (g != f && inexact) atomicAdd(inexact, 1);
    }
    const int64_t tile = row / TILE_ROWS * chunks + o / 8;
    wt[tile * TILE_BYTES + TILE_W + (row % TILE_ROWS) * 8 + o % 8] = v;
  }
}

int sms() {
  int dev = 0, n = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

// CTAs of a call: one per SM, more when a CTA would stage more than LMAX
// K chunks of tokens, never more than tiles.
int64_t grid_of(int64_t tiles) {
  return std::min<int64_t>(tiles, std::max<int64_t>(sms(), (tiles + LMAX - 1) / LMAX));
}

int sticky_w4(int* out, int clear, cudaStream_t st) { return tc::sticky_read(out, clear, st); }

}  // namespace w4
}  // namespace vq

using namespace vq::w4;

extern "C" {

int64_t vq_w4_packed_bytes(int64_t N, int64_t K) {
  if (N <= 0 || K <= 0 || K % 128) return -1;
  return (N + TILE_ROWS - 1) / TILE_ROWS * (K / 128) * TILE_BYTES;
}

int64_t vq_w4a8_workspace_bytes(int64_t N, int64_t K) {
  if (N <= 0 || K <= 0 || K % 128) return -1;
  return (N + TILE_ROWS - 1) / TILE_ROWS * TILE_ROWS * 16 * (int64_t)sizeof(float);
}

int vq_w4_pack_weights(const vq_tensor* codes, const vq_tensor* scales, void* packed,
                       int32_t* d_inexact, void* stream) {
  if (!codes || !scales || !packed) return VQ_ERR_NULL;
  if (codes->dtype != VQ_BF16 || scales->dtype != VQ_BF16) return VQ_ERR_UNSUPPORTED;
  if (codes->ndim != 2 || scales->ndim != 2) return VQ_ERR_SHAPE;
  const int64_t N = codes->shape[0], K = codes->shape[1];
  if (K % 128 || N <= 0 || scales->shape[0] != N || scales->shape[1] != K / 16) return VQ_ERR_SHAPE;
  if (vq_w4_packed_bytes(N, K) >= (1ll << 31)) return VQ_ERR_UNSUPPORTED;
  if (reinterpret_cast<uintptr_t>(packed) & 15) return VQ_ERR_ALIGNMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (d_inexact && cudaMemsetAsync(d_inexact, 0, 4, st) != cudaSuccess) return VQ_ERR_CUDA;
  const int64_t n = (N + TILE_ROWS - 1) / TILE_ROWS * TILE_ROWS * (K / 2);
  k_w4_pack<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(
      (const uint16_t*)codes->data, (const uint16_t*)scales->data, (uint8_t*)packed, (int)N,
      (int)K, d_inexact);
  return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
}

int vq_w4a8_linear_small(const vq_tensor* a_codes, const vq_tensor* a_scales, const void* packed,
                         int64_t N, const void* bias, float* workspace, int32_t* counters,
                         int32_t* d_err, void* out, void* stream) {
  if (!a_codes || !a_scales || !packed || !workspace || !counters || !out) return VQ_ERR_NULL;
  if (a_codes->dtype != VQ_BF16 || a_scales->dtype != VQ_BF16) return VQ_ERR_UNSUPPORTED;
  if (a_codes->ndim != 2 || a_scales->ndim != 2) return VQ_ERR_SHAPE;
  const int64_t M = a_codes->shape[0], K = a_codes->shape[1];
  if (a_scales->shape[0] != M || a_scales->shape[1] != K / 32) return VQ_ERR_SHAPE;
  if (M <= 0 || M > 16 || N <= 0 || K <= 0 || K % 128) return VQ_ERR_UNSUPPORTED;
  if (vq_w4_packed_bytes(N, K) >= (1ll << 31)) return VQ_ERR_UNSUPPORTED;
  const void* ptrs[3] = {a_codes->data, packed, workspace};
  for (const void* q : ptrs)
    if (reinterpret_cast<uintptr_t>(q) & 15) return VQ_ERR_ALIGNMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (d_err && cudaMemsetAsync(d_err, 0, sizeof(int32_t), st) != cudaSuccess) return VQ_ERR_CUDA;
  Args p;
  p.wt = (const uint8_t*)packed;
  p.ac = (const uint16_t*)a_codes->data;
  p.as = (const uint16_t*)a_scales->data;
  p.bias = (const uint16_t*)bias;
  p.out = (uint16_t*)out;
  p.acc = workspace;
  p.done = counters;
  p.err = d_err;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.chunks = (int)(K / 128);
  const int64_t tiles = (N + TILE_ROWS - 1) / TILE_ROWS * p.chunks;
  p.tiles = (int)tiles;
  p.G = (int)grid_of(tiles);
  // the kernel's tile ranges are 32-bit unsigned products (always true for
  // packed weights below 2 GB: T <= 2^17, G <= max(SMs, T / LMAX))
  if (tiles * p.G >= (1ll << 32)) return VQ_ERR_UNSUPPORTED;
  // a CTA stages at most ceil(T / G) <= LMAX chunks of tokens
  const int L = (int)std::min<int64_t>((tiles + p.G - 1) / p.G, p.chunks);
  // programmatic dependent launch: the kernel may start while the previous
  // grid on the stream finishes, streaming its (constant) weights at once
  auto kern = M <= 8 ? k_w4a8<1> : k_w4a8<2>;
  const int smem = smem_bytes(M <= 8 ? 1 : 2, L);
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return VQ_ERR_CUDA;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)p.G);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, p) != cudaSuccess) return VQ_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
}

}  // extern "C"
