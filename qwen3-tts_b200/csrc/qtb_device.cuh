// qtb_device.cuh -- device-side helpers shared by every sm_100a kernel of the
// decode engine: PTX wrappers (streaming loads, mma.sync, bulk copies,
// mbarriers), bf16/fp16 bit tricks, warp reductions and the bounded grid
// barrier used by the persistent decode kernel.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#define QTB_DEV __device__ __forceinline__
#define QTB_HOST_DEV __host__ __device__ __forceinline__

namespace qtb {

// ---------------------------------------------------------------- loads ----
// Weights, norm gains, RoPE tables, embedding tables and page tables are
// read-only for a kernel's lifetime: non-coherent path, no L1 allocation.
QTB_DEV uint4 ld_stream(const void *p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}
// Same, with an L2 eviction-priority policy (created once per thread).
QTB_DEV uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
QTB_DEV uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
QTB_DEV uint4 ld_stream_hint(const void *p, uint64_t pol) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p), "l"(pol));
  return r;
}
QTB_DEV uint2 ld_nc_u2(const void *p) {
  uint2 r;
  asm volatile("ld.global.nc.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
  return r;
}
QTB_DEV uint4 ld_nc_u4(const void *p) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}
// Activations, partial sums and KV pages are produced by other CTAs inside the
// same persistent launch: read them at L2 (".cg") so a stale L1 line is never
// used.
QTB_DEV float ld_cg(const float *p) { return __ldcg(p); }
QTB_DEV float4 ld_cg4(const float *p) { return __ldcg(reinterpret_cast<const float4 *>(p)); }
QTB_DEV uint4 ld_cg_u4(const void *p) { return __ldcg(reinterpret_cast<const uint4 *>(p)); }

// ------------------------------------------------------------- numerics ----
QTB_DEV float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
QTB_DEV float bf16hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
// f32 -> bf16 by truncation (the reference's KV store semantics, bits >> 16).
QTB_DEV uint32_t f32_to_bf16_trunc(float f) { return __float_as_uint(f) >> 16; }
// f32 -> bf16 round-to-nearest-even (used only to split activations into
// hi + lo bf16 parts for the tensor-core GEMV).
QTB_DEV uint32_t f32_to_bf16_rn(float f) {
  uint32_t u = __float_as_uint(f);
  u += 0x7fffu + ((u >> 16) & 1u);
  return u >> 16;
}
QTB_DEV float half_bits_to_f32(uint32_t h) { return __half2float(__ushort_as_half((unsigned short)h)); }

// Orderable key for a float: larger float <=> larger unsigned key.
QTB_DEV uint32_t float_order_key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

template <typename T>
QTB_DEV T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
QTB_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---------------------------------------------------------- tensor cores ---
// D(16x8,f32) += A(16x16) * B(16x8); A row-major fragment (4 regs), B column
// fragment (2 regs).  The GEMV keeps weights as A and the activation (split
// into hi and lo halves, one per column) as B.
QTB_DEV void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
QTB_DEV void mma_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// D(16x8,s32) += A(16x32,s8) * B(32x8,s8), exact integer accumulation.
// A: 4 regs (rows gid / gid+8, k 4tig..4tig+3 and 16+4tig..), B: 2 regs
// (k 4tig..4tig+3 and 16+4tig.., column gid).
QTB_DEV void mma_s8(int (&d)[4], const uint4 &a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
}

// Two signed int8 weights (selected bytes of w, already XOR 0x80) -> f16x2
// holding exactly their values: 0x64XX is 1024 + XX in fp16.
QTB_DEV uint32_t i8x2_to_f16x2(uint32_t w_xor80, uint32_t sel) {
  uint32_t h = __byte_perm(w_xor80, 0x00006464u, sel);
  const uint32_t bias = 0x64806480u;  // (1024 + 128, 1024 + 128)
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(h), "r"(bias));
  return r;
}
// Two 4-bit codes (bits [0,4) and [16,20) of w) -> f16x2 holding the codes.
QTB_DEV uint32_t u4x2_to_f16x2(uint32_t w) {
  uint32_t h = (w & 0x000f000fu) | 0x64006400u;
  const uint32_t bias = 0x64006400u;  // (1024, 1024)
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(h), "r"(bias));
  return r;
}

// -------------------------------------------------- bulk copies (TMA 1D) ---
QTB_DEV uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
QTB_DEV void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
QTB_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
QTB_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
QTB_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
QTB_DEV void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
QTB_DEV void bulk_g2s(void *dst_smem, const void *src_gmem, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// Tiled TMA load of a 3-D box (no multicast): coordinates x (innermost,
// elements), y, z of the tensor map at generic address `map` (global memory).
QTB_DEV void tma_load_3d(void *dst_smem, const void *map, int x, int y, int z, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          smem_u32(dst_smem)),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}
// Four transposed 8 x 8 b16 matrices from shared memory (lane 8i + r gives
// row r of matrix i).
QTB_DEV void ldsm_x4_trans(uint32_t (&r)[4], const void *row_addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(row_addr))
               : "memory");
}
QTB_DEV void bulk_g2s_hint(void *dst_smem, const void *src_gmem, uint32_t bytes, uint64_t *bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}
// Bounded wait on an mbarrier phase. Returns false after ~`limit_cycles`.
QTB_DEV bool mbar_wait(uint64_t *bar, uint32_t parity, long long limit_cycles) {
  uint32_t done = 0;
  long long t0 = clock64();
  while (true) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (done) return true;
    if (clock64() - t0 > limit_cycles) return false;
  }
}

// Named barrier `id` over `nthreads` threads (whole warps, warp-uniform call).
QTB_DEV void bar_sync_n(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
// ... that also returns the AND of `v` over the participating threads.
QTB_DEV bool bar_and_n(int id, int nthreads, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "bar.red.and.pred p, %2, %3, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

// Non-blocking probe of an mbarrier phase (true once the phase of the given
// parity has completed).
QTB_DEV bool mbar_test(uint64_t *bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}
// Ask L2 to fetch [p, p + bytes) (16-byte aligned, multiple of 16 bytes);
// nothing waits for it.
QTB_DEV void prefetch_l2(const void *p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Distributed shared memory: the address of `p` (this CTA's shared memory) in
// CTA `rank` of the cluster, a store there, and a remote mbarrier arrive whose
// release orders this thread's earlier cluster stores.
QTB_DEV uint32_t cluster_map(const void *p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
QTB_DEV void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
QTB_DEV void mbar_arrive_remote(uint32_t bar_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_addr) : "memory");
}
// Bounded wait on a local mbarrier phase completed by another CTA of the
// cluster (acquire at cluster scope makes its stores visible).
QTB_DEV bool mbar_wait_cluster(uint64_t *bar, uint32_t parity, long long limit_cycles) {
  uint32_t done = 0;
  const long long t0 = clock64();
  while (true) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (done) return true;
    if (clock64() - t0 > limit_cycles) return false;
  }
}

// ----------------------------------------------- 5th-gen tensor cores ------
// tcgen05: MMAs issued by one thread read both operands from shared memory
// through 64-bit matrix descriptors and accumulate into tensor memory (TMEM,
// 128 lanes x 512 32-bit columns per SM); completion is signalled through an
// mbarrier (tcgen05.commit); the accumulator is read back with tcgen05.ld,
// warp w of the CTA seeing lanes 32 (w % 4) .. 32 (w % 4) + 31.

// Allocate `ncols` TMEM columns (power of two >= 32); the base address is
// written to shared memory.  Whole warp.
QTB_DEV void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
QTB_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
QTB_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
QTB_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor of a K-major operand tile in the 128-byte
// swizzled canonical layout: rows of 128 bytes (one K chunk), 8-row groups of
// 1024 bytes (stride byte offset), the 16-byte units of row r XOR-permuted by
// r % 8.  The tile base is 1024-byte aligned; moving along K inside the
// 128-byte row adds the byte offset to the start address.
QTB_DEV uint64_t umma_desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3fffu)      // start address
         | ((uint64_t)1u << 16)                  // leading byte offset (unused with this swizzle)
         | ((uint64_t)(1024u >> 4) << 32)        // stride byte offset: 8 rows x 128 B
         | ((uint64_t)1u << 46)                  // descriptor version (sm_100)
         | ((uint64_t)2u << 61);                 // 128-byte swizzle
}
// Instruction descriptor: D format (1 f32, 2 s32), A/B formats (kind::f16:
// 1 = bf16; kind::i8: 1 = s8), both K-major, N and M = 128.
QTB_HOST_DEV constexpr uint32_t umma_idesc(uint32_t dfmt, uint32_t abfmt, uint32_t n) {
  return (dfmt << 4) | (abfmt << 7) | (abfmt << 10) | ((n >> 3) << 17) | ((128u >> 4) << 24);
}
// D[tmem] (+)= A[128 x 32 B of K] * B[N x 32 B of K]^T; accumulate = 0 overwrites.
QTB_DEV void umma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
QTB_DEV void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` once every tcgen05 operation this thread issued before has
// completed (their shared-memory reads included).
QTB_DEV void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
// 32 consecutive 32-bit TMEM columns of this thread's lane, then wait.
QTB_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

QTB_DEV unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ------------------------------------------------------------ grid sync ----
QTB_DEV unsigned ld_acquire_gpu(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Two adjacent 32-bit words (8-byte aligned) read by one acquire load.
QTB_DEV uint2 ld_acquire_gpu_v2(const unsigned *p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return make_uint2((unsigned)v, (unsigned)(v >> 32));
}
QTB_DEV unsigned atom_add_acq_rel_gpu(unsigned *p, unsigned v) {
  unsigned old;
  asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
QTB_DEV unsigned atom_add_release_gpu(unsigned *p, unsigned v) {
  unsigned old;
  asm volatile("atom.add.release.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
QTB_DEV void st_release_gpu(unsigned *p, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

}  // namespace qtb
