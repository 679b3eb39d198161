// Thin inline-PTX wrappers for sm_100a: mbarrier, TMA (cp.async.bulk.tensor), tcgen05
// (alloc / mma.block_scale / cp / commit / ld), cluster helpers.  No library dependencies.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace qk {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ bool elect_one() {
  uint32_t pred;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// ------------------------------------------------------------------ cluster -------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t num_clusters_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// shared::cta address of this CTA -> shared::cluster address of the same offset in `rank`
__device__ __forceinline__ uint32_t mapa(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

// ------------------------------------------------------------------ mbarrier ------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// arrive on a barrier given by a shared::cluster address (own or peer CTA), releasing this thread's earlier
// memory operations at cluster scope: for hand-offs of data written to a peer's shared memory
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster_addr)
               : "memory");
}
// the same arrive with CTA-scope release: for hand-offs of tensor memory, where the ordering comes from
// tcgen05.wait::ld / tcgen05.fence::before_thread_sync and no shared or global data changes hands.  (The
// cluster-scope release above drains the thread's outstanding stores first: measured 1.8k cycles per arrive in
// an epilogue warp, which delayed the next tile's first MMA by that much.)
__device__ __forceinline__ void mbar_arrive_remote(uint32_t bar_cluster_addr) {
  asm volatile("mbarrier.arrive.release.cta.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster_addr) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
// try_wait suspends the thread in hardware until the phase completes or the hint (ns) runs
// out; a generous hint keeps waiting warps from re-polling (they wake at once on completion).
constexpr uint32_t kSuspendHintNs = 20000;
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return done != 0;
}
// cluster-scope acquire variant: used when the arrivals come from the peer CTA
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return done != 0;
}

// ------------------------------------------------------------------ fences --------------
// ---- programmatic dependent launch ----
// launch_dependents: the next kernel of the stream (if it was launched with programmatic stream
// serialisation) may start its CTAs once every CTA of this grid has executed this (or exited).
// wait: returns when the preceding grid has completed and its memory is visible; a kernel launched
// without a programmatic predecessor passes straight through.
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---- cluster launch control (dynamic tile scheduler) ----
// Asks the hardware to cancel the launch of a cluster of this grid that has not started yet; the
// 16-byte answer lands in `resp` (shared memory of this CTA) and completes 16 bytes on `bar`.
__device__ __forceinline__ void clc_try_cancel(uint32_t resp, uint32_t bar) {
  asm volatile("clusterlaunchcontrol.try_cancel.async.shared::cta.mbarrier::complete_tx::bytes.b128 [%0], [%1];" ::"r"(resp),
               "r"(bar)
               : "memory");
}
// Decodes an answer: blockIdx.x of the first CTA of the cancelled cluster, or -1 when nothing
// was left to cancel (after which this cluster must not ask again).
__device__ __forceinline__ int clc_query_first_ctaid_x(uint32_t resp) {
  uint32_t x, valid;
  asm volatile(
      "{\n"
      ".reg .pred p1;\n"
      ".reg .b128 r;\n"
      "ld.shared.b128 r, [%2];\n"
      "clusterlaunchcontrol.query_cancel.is_canceled.pred.b128 p1, r;\n"
      "selp.u32 %1, 1, 0, p1;\n"
      "mov.u32 %0, 0;\n"
      "@p1 clusterlaunchcontrol.query_cancel.get_first_ctaid::x.b32.b128 %0, r;\n"
      "}\n"
      : "=r"(x), "=r"(valid)
      : "r"(resp)
      : "memory");
  return valid ? static_cast<int>(x) : -1;
}
__device__ __forceinline__ void st_shared_cluster_u32(uint32_t cluster_addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ------------------------------------------------------------------ TMA -----------------
__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}
// 2-D tiled load, completion on an mbarrier of this CTA
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* tmap, uint32_t bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void* tmap, uint32_t bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
// CTA-pair forms: data lands in this CTA's smem, the transaction bytes are signalled on an
// mbarrier that may live in the peer CTA (bar is a shared::cluster address).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const void* tmap, uint32_t bar_cluster, int c0,
                                                 int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar_cluster), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const void* tmap, uint32_t bar_cluster, int c0,
                                                 int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar_cluster), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
// L2 prefetch of the box a later tiled load will fetch (no shared-memory destination)
__device__ __forceinline__ void tma_prefetch_2d(const void* tmap, int c0, int c1) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(reinterpret_cast<uint64_t>(tmap)),
               "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void tma_prefetch_3d(const void* tmap, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                   reinterpret_cast<uint64_t>(tmap)),
               "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void tma_store_2d(const void* tmap, uint32_t src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(tmap)),
               "r"(src), "r"(c0), "r"(c1)
               : "memory");
}
// Untiled bulk copy (both addresses 16-byte aligned, size a multiple of 16 bytes):
// this CTA's shared memory -> global, tracked by the thread's bulk async-groups (tma_store_commit / _wait)
__device__ __forceinline__ void bulk_store(void* dst, uint32_t src_smem, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(reinterpret_cast<uint64_t>(dst)),
               "r"(src_smem), "r"(bytes)
               : "memory");
}
// per-thread asynchronous 16-byte copy global -> shared (load/store unit, not the bulk copy unit)
__device__ __forceinline__ void cp_async_16(uint32_t dst_smem, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst_smem), "l"(reinterpret_cast<uint64_t>(src)) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// stores through an NVSwitch multicast mapping: the switch writes the value into the memory of every GPU bound to it
__device__ __forceinline__ void multimem_st_v4(void* mc_addr, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(reinterpret_cast<uint64_t>(mc_addr)),
               "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void multimem_st_u32(void* mc_addr, uint32_t v) {
  asm volatile("multimem.st.relaxed.sys.global.u32 [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(mc_addr)), "r"(v) : "memory");
}
__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(reinterpret_cast<uint64_t>(p)));
  return v;
}
// orders this thread's generic-proxy accesses against its asynchronous-proxy ones (every state space)
__device__ __forceinline__ void fence_proxy_async_all() { asm volatile("fence.proxy.async;" ::: "memory"); }

__device__ __forceinline__ void tma_store_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void tma_store_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
template <int N>
__device__ __forceinline__ void tma_store_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// ------------------------------------------------------------------ TMEM ----------------
template <int CG>
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  if constexpr (CG == 1)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
                 : "memory");
  else
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
                 : "memory");
}
template <int CG>
__device__ __forceinline__ void tmem_relinquish() {
  if constexpr (CG == 1)
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  else
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
template <int CG>
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  if constexpr (CG == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
  else
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// The tcgen05 wrappers below take the two 32-bit halves of a shared-memory descriptor, which keeps the
// descriptor arithmetic in 32-bit, warp-uniform registers.
//
// tcgen05.cp 32x128b.warpx4: shared memory -> tensor memory copy of one 512-byte scale-factor atom (32 rows
// x 16 bytes), replicated into the four 32-lane sub-partitions, 4 TMEM columns wide.
//
// tcgen05.mma ... block_scale: D[tmem] (+)= A[smem] * B[smem] with per-block scale factors read from TMEM.
// KIND 0: kind::mxf8f6f4 (E8M0 scales, one per 32 K); KIND 1: kind::mxf4nvf4 with one E4M3 scale per 16 K
// (scale_vec::4X, NVFP4); KIND 2: kind::mxf4nvf4 with one E8M0 scale per 32 K (scale_vec::2X, MXFP4).
template <int CG>
__device__ __forceinline__ void tc_cp_32x128b_warpx4_lh(uint32_t taddr, uint32_t lo, uint32_t hi) {
  if constexpr (CG == 1)
    asm volatile("{\n\t.reg .b64 d;\n\tmov.b64 d, {%1, %2};\n\ttcgen05.cp.cta_group::1.32x128b.warpx4 [%0], d;\n\t}" ::"r"(taddr),
                 "r"(lo), "r"(hi)
                 : "memory");
  else
    asm volatile("{\n\t.reg .b64 d;\n\tmov.b64 d, {%1, %2};\n\ttcgen05.cp.cta_group::2.32x128b.warpx4 [%0], d;\n\t}" ::"r"(taddr),
                 "r"(lo), "r"(hi)
                 : "memory");
}

#define QK_MMA_BS_ASM(CGSTR, KINDSTR)                                                                              \
  asm volatile(                                                                                                    \
      "{\n\t.reg .pred p;\n\t.reg .b64 da, db;\n\tsetp.ne.b32 p, %6, 0;\n\tmov.b64 da, {%1, %2};\n\tmov.b64 db, {%3, %4};\n\t" \
      "tcgen05.mma.cta_group::" CGSTR ".kind::" KINDSTR " [%0], da, db, %5, [%7], [%8], p;\n\t}" ::"r"(d_tmem),      \
      "r"(a_lo), "r"(a_hi), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)          \
      : "memory")

template <int KIND, int CG>
__device__ __forceinline__ void tc_mma_block_scale_lh(uint32_t d_tmem, uint32_t a_lo, uint32_t a_hi, uint32_t b_lo,
                                                      uint32_t b_hi, uint32_t idesc, uint32_t sfa_tmem,
                                                      uint32_t sfb_tmem, uint32_t accumulate) {
  if constexpr (KIND == 0) {
    if constexpr (CG == 1) QK_MMA_BS_ASM("1", "mxf8f6f4.block_scale");
    else QK_MMA_BS_ASM("2", "mxf8f6f4.block_scale");
  } else if constexpr (KIND == 1) {
    if constexpr (CG == 1) QK_MMA_BS_ASM("1", "mxf4nvf4.block_scale.scale_vec::4X");
    else QK_MMA_BS_ASM("2", "mxf4nvf4.block_scale.scale_vec::4X");
  } else {
    if constexpr (CG == 1) QK_MMA_BS_ASM("1", "mxf4nvf4.block_scale.scale_vec::2X");
    else QK_MMA_BS_ASM("2", "mxf4nvf4.block_scale.scale_vec::2X");
  }
}
#undef QK_MMA_BS_ASM

// Shared-memory matrix descriptors, as (low, high) 32-bit halves.
//   K-major operand tile stored with the 128-byte swizzle (rows of 128 bytes, 8-row groups 1024 bytes apart):
//     low  = start address in 16-byte units | leading byte offset 1 (unused with swizzle) << 16
//     high = stride byte offset (1024 >> 4) | descriptor version 1 << 14 | layout SWIZZLE_128B (2) << 29
//   unswizzled 512-byte scale-factor atom (32 rows x 16 bytes; 8-row core matrices 128 bytes apart):
//     low  = start address in 16-byte units;  high = stride byte offset (128 >> 4) | version 1 << 14
__device__ __forceinline__ uint32_t sdesc_lo_sw128(uint32_t saddr) { return ((saddr & 0x3FFFFu) >> 4) | (1u << 16); }
constexpr uint32_t kSdescHiSw128 = (1024u >> 4) | (1u << 14) | (2u << 29);
__device__ __forceinline__ uint32_t sdesc_lo_sf(uint32_t saddr) { return (saddr & 0x3FFFFu) >> 4; }
constexpr uint32_t kSdescHiSf = (128u >> 4) | (1u << 14);

// Make an mbarrier track completion of all tcgen05 ops this thread issued so far.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
// CTA-pair form: arrives on the barrier at the same offset in every CTA of `mask`.
__device__ __forceinline__ void tc_commit_pair(uint32_t bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
      "h"(mask)
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns -> 32 registers per thread (thread = lane = row)
__device__ __forceinline__ void tc_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ------------------------------------------------------------------ descriptors ---------
// Instruction descriptor of the block-scaled MMA.
//   [4,6) B scale id  [7,10) A format  [10,13) B format  [15] A major  [16] B major
//   [17,23) N>>3  [23] scale format (0 E4M3, 1 E8M0)  [24,29) M>>4  [29,31) A scale id
// Element formats: kind::mxf8f6f4 E4M3 = 0, E5M2 = 1 (given per operand by `a_fmt` / `b_fmt`);
// kind::mxf4nvf4 E2M1 = 1.
__host__ __device__ constexpr uint32_t make_idesc_block_scaled(int kind, int mma_m, int mma_n, uint32_t a_fmt = 0,
                                                                uint32_t b_fmt = 0) {
  uint32_t d = 0;
  d |= (kind == 0 ? a_fmt : 1u) << 7;
  d |= (kind == 0 ? b_fmt : 1u) << 10;
  d |= static_cast<uint32_t>(mma_n >> 3) << 17;
  d |= (kind == 1 ? 0u : 1u) << 23;
  d |= static_cast<uint32_t>(mma_m >> 4) << 24;
  return d;
}
__device__ __forceinline__ uint32_t idesc_with_sf_id(uint32_t idesc, uint32_t a_id, uint32_t b_id) {
  return idesc | (b_id << 4) | (a_id << 29);
}

}  // namespace qk
