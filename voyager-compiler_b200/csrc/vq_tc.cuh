// Building blocks shared by the tcgen05 kernels (MXFP8 GEMM, MXFP8
// attention): mbarriers with bounded waits, TMA / bulk copies (never with
// cluster multicast), shared-memory and instruction descriptors for
// tcgen05.mma.kind::mxf8f6f4.block_scale, and the tensor-map encoder.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace vq {
namespace tc {

constexpr uint64_t WAIT_NS = 2000000000ull;  // a wait gives up after 2 s

// The first wait-timeout code that any kernel of this translation unit
// recorded on this device since it was last cleared: the per-call error
// words tell one caller about its own launch, this word lets the host ask
// afterwards whether any launch gave up (vq_device_errors).  One copy per
// translation unit that includes this header.
static __device__ int g_sticky_err;

// Record a wait that gave up: the launch's own error word and the sticky one.
__device__ __forceinline__ void note_err(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
  atomicCAS(&g_sticky_err, 0, code);
}

// Host side: read (and with clear, reset) this translation unit's sticky
// word on the current device; synchronises `st`.
static inline int sticky_read(int* out, int clear, cudaStream_t st) {
  int v = 0;
  if (cudaMemcpyFromSymbolAsync(&v, g_sticky_err, sizeof(int), 0, cudaMemcpyDeviceToHost, st) !=
          cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return -1;
  if (clear && v) {
    const int z = 0;
    if (cudaMemcpyToSymbolAsync(g_sticky_err, &z, sizeof(int), 0, cudaMemcpyHostToDevice, st) !=
            cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
      return -1;
  }
  *out = v;
  return 0;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait: false (and *err set to code) if the phase has not completed
// within WAIT_NS of wall-clock time.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > WAIT_NS) break;
  }
  note_err(err, code);
  return false;
}

// mbar_wait by every lane of a warp, with one outcome for the whole warp (a
// warp that goes on to a .sync.aligned tcgen05 instruction must not split).
__device__ __forceinline__ bool mbar_wait_warp(uint32_t bar, uint32_t parity, int* err, int code) {
  return __all_sync(0xFFFFFFFFu, mbar_wait(bar, parity, err, code)) != 0;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
      "%3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// K-major SWIZZLE_128B shared-memory matrix descriptor (tcgen05 format,
// version 1): start >> 4, LBO 1 (unused for swizzled K-major), SBO = 1024 B
// between 8-row groups, layout type 2.  Rows are 128 bytes; the 16-byte
// chunk c of row r sits at r * 128 + ((c ^ (r % 8)) * 16) of a
// 1024-byte-aligned tile.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;  // version
  d |= (uint64_t)2 << 61;  // SWIZZLE_128B
  return d;
}
// Descriptor of a 32-row x 16-byte scale atom for tcgen05.cp.32x128b:
// no swizzle, 8-row core matrices 128 B apart.
__device__ __forceinline__ uint64_t sf_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(128 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  return d;
}

// Instruction descriptor, kind::mxf8f6f4 block-scaled: E4M3 x E4M3, UE8M0
// scales, K-major A and B, M x N, scale-factor byte j of A and of B.
__device__ __forceinline__ uint32_t idesc_mxf8(uint32_t j, uint32_t M, uint32_t N) {
  return (j << 4) | (0u << 7) | (0u << 10) | ((N >> 3) << 17) | (1u << 23) | ((M >> 4) << 24) |
         (j << 29);
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

// One block-scaled MMA: D (+)= A . B^T with the scale vectors at sfa / sfb
// (TMEM), K = 32.
__device__ __forceinline__ void mma_mxf8(uint32_t d_tmem, uint64_t da, uint64_t db, uint32_t idesc,
                                         uint32_t accum, uint32_t sfa_tmem, uint32_t sfb_tmem) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], "
      "p;\n\t}" ::"r"(d_tmem),
      "l"(da), "l"(db), "r"(idesc), "r"(accum), "r"(sfa_tmem), "r"(sfb_tmem));
}
// 128 lanes x 16 bytes of scale factors from shared memory into TMEM.
__device__ __forceinline__ void cp_sf(uint32_t tmem_col, uint32_t saddr) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(tmem_col),
               "l"(sf_desc(saddr)));
}
// Arrive on an mbarrier once every tcgen05 operation this thread issued so
// far has completed.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}

// 32 consecutive fp32 columns of this warp's 32 TMEM lanes (lane = thread).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---- CTA pairs (tcgen05 cta_group::2) ---------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// The shared::cluster address of the same shared variable in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
// TMA tile load into this CTA's shared memory whose completion is counted on
// an mbarrier of either CTA of the pair (no multicast).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int x, int y,
                                                 uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar_cluster)
      : "memory");
}
// Pair MMA (issued by the even CTA): D (+)= A . B^T over both CTAs' shared
// memory (same offsets), each CTA's TMEM holding its half of the rows.
__device__ __forceinline__ void mma_mxf8_pair(uint32_t d_tmem, uint64_t da, uint64_t db,
                                              uint32_t idesc, uint32_t accum, uint32_t sfa_tmem,
                                              uint32_t sfb_tmem) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], "
      "p;\n\t}" ::"r"(d_tmem),
      "l"(da), "l"(db), "r"(idesc), "r"(accum), "r"(sfa_tmem), "r"(sfb_tmem));
}
// The same, accumulating (D += A . B^T).
__device__ __forceinline__ void mma_mxf8_pair_acc(uint32_t d_tmem, uint64_t da, uint64_t db,
                                                  uint32_t idesc, uint32_t sfa_tmem,
                                                  uint32_t sfb_tmem) {
  asm volatile(
      "tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%4], [%5], 1;" ::"r"(
          d_tmem),
      "l"(da), "l"(db), "r"(idesc), "r"(sfa_tmem), "r"(sfb_tmem));
}
// Scale atoms of both CTAs (same shared offset) into their own TMEM, from a
// prepared descriptor (sf_desc).
__device__ __forceinline__ void cp_sf_pair_desc(uint32_t tmem_col, uint64_t desc) {
  asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" ::"r"(tmem_col), "l"(desc));
}
// A shared-memory descriptor moved by off16 x 16 bytes: the start address
// field is the low 14 bits (address / 16); for shared addresses below 2^18
// the sum stays inside the field, so only the low word changes.
__device__ __forceinline__ uint64_t desc_at(uint64_t d0, uint32_t off16) {
  return (d0 & 0xFFFFFFFF00000000ull) | (uint32_t)((uint32_t)d0 + off16);
}
// Arrive on the mbarrier at this offset in the CTAs of `mask` once the pair's
// tcgen05 operations issued so far have completed.
__device__ __forceinline__ void tc_commit_pair(uint32_t bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
      "[%0], %1;" ::"r"(bar),
      "h"(mask)
      : "memory");
}

}  // namespace tc

namespace mx {
// A 2-D uint8 tensor map over [rows, cols_bytes] (row stride cols_bytes)
// with a box of 128 bytes x box_rows rows, SWIZZLE_128B (defined in
// vq_gemm.cu).
bool make_map(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols_bytes,
              uint32_t box_rows);
// Same without swizzle and with a box of box_cols bytes x box_rows rows.
bool make_map_plain(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols_bytes,
                    uint32_t box_cols, uint32_t box_rows);
int sm_count();
}  // namespace mx
}  // namespace vq
