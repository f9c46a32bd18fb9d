// Blackwell (sm_100a) building blocks: tcgen05 tensor-core MMAs with TMEM
// accumulators, TMA tile loads, mbarriers with bounded waits.
//
// Operand tiles in shared memory use the 128-byte swizzled layout that TMA
// writes with CU_TENSOR_MAP_SWIZZLE_128B: a tile of R rows x 64 bf16 columns
// is R x 128 bytes, and the 16-byte piece p of row r sits at piece p ^ (r % 8).
// Tiles start on 1024-byte boundaries (one swizzle atom = 8 rows).
//
// Descriptor encodings follow the public sm100 UMMA descriptor definitions
// (CUTLASS cute/arch/mma_sm100_desc.hpp):
//   shared-memory descriptor: start >> 4 in bits [0,14), leading byte offset
//   >> 4 in [16,30), stride byte offset >> 4 in [32,46), version 1 in
//   [46,48), layout type in [61,64) (2 = SWIZZLE_128B);
//   instruction descriptor (kind::f16): D format [4,6) (1 = f32), A format
//   [7,10) and B format [10,13) (1 = bf16), A major bit 15, B major bit 16
//   (0 = K-major, 1 = MN-major), N >> 3 in [17,23), M >> 4 in [24,29).
//   K-major SW128: rows of 128 bytes, 8-row groups 1024 bytes apart (SBO),
//   one K step of 16 bf16 = +32 bytes of start address.
//   MN-major SW128: 64 MN elements per 128-byte row, K rows 128 bytes apart,
//   8-K-row groups SBO apart, 64-element MN blocks LBO apart.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace gdn2 {
namespace tc {

// ---------------------------------------------------------------------------
// addresses
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Every wait in these kernels gives up after this long and reports it.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

// ---------------------------------------------------------------------------
// mbarriers
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// The waiting thread is suspended in hardware until the phase completes or
// the hint (ns) runs out, so waiting warps take no issue slots from the rest.
constexpr uint32_t kSuspendHintNs = 10000000u;

__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(addr), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity to complete; false after
// kWaitLimitNs (the caller records the timeout and abandons its work).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(addr, parity)) return true;
    if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
  }
}

// ---------------------------------------------------------------------------
// TMA (no multicast) and bulk copies
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// pulls one box of a tensor map into L2 (no shared memory, no completion to wait for)
__device__ __forceinline__ void tma_prefetch_3d(const CUtensorMap* map, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}

__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap* map, int c0, int c1) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1)
               : "memory");
}

// contiguous global -> shared copy; both addresses 16-byte aligned, bytes % 16 == 0
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// shared -> global tile store (the source must have been made visible to the
// async proxy with fence_proxy_async by every thread that wrote it)
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// the sources of every committed store group have been read (smem reusable)
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// every committed store group has completed (writes visible in global memory)
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// generic-proxy shared-memory writes -> visible to the async proxy (MMA, TMA)
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// TMEM
// ---------------------------------------------------------------------------
// whole warp; the allocated base address is written to *slot
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t base, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane (32x32b shape: warp
// w % 4 reads lanes [32 (w % 4), 32 (w % 4) + 32), thread i lane 32 (w % 4) + i)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&x)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) x[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&x)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(x[0])), "r"(__float_as_uint(x[1])), "r"(__float_as_uint(x[2])),
      "r"(__float_as_uint(x[3])), "r"(__float_as_uint(x[4])), "r"(__float_as_uint(x[5])),
      "r"(__float_as_uint(x[6])), "r"(__float_as_uint(x[7])), "r"(__float_as_uint(x[8])),
      "r"(__float_as_uint(x[9])), "r"(__float_as_uint(x[10])), "r"(__float_as_uint(x[11])),
      "r"(__float_as_uint(x[12])), "r"(__float_as_uint(x[13])), "r"(__float_as_uint(x[14])),
      "r"(__float_as_uint(x[15])), "r"(__float_as_uint(x[16])), "r"(__float_as_uint(x[17])),
      "r"(__float_as_uint(x[18])), "r"(__float_as_uint(x[19])), "r"(__float_as_uint(x[20])),
      "r"(__float_as_uint(x[21])), "r"(__float_as_uint(x[22])), "r"(__float_as_uint(x[23])),
      "r"(__float_as_uint(x[24])), "r"(__float_as_uint(x[25])), "r"(__float_as_uint(x[26])),
      "r"(__float_as_uint(x[27])), "r"(__float_as_uint(x[28])), "r"(__float_as_uint(x[29])),
      "r"(__float_as_uint(x[30])), "r"(__float_as_uint(x[31]))
      : "memory");
}

// M = 64 accumulators (cta_group::1) keep row m in TMEM lane 32 (m / 16) + m % 16;
// warp w reads rows [16 (w % 4), 16 (w % 4) + 16) of its lane quarter.  The
// 16x256b shape hands each thread exactly the m16n8 accumulator fragment of
// mma.sync: per 8-column group j, registers {4j, 4j+1} = row g, columns 2t, 2t+1
// and {4j+2, 4j+3} = row g + 8 (g = lane / 4, t = lane % 4).  NF groups of 8
// columns starting at the address's column.
template <int NF>
__device__ __forceinline__ void tmem_ld_frag(uint32_t taddr, float (*f)[4]);

template <>
__device__ __forceinline__ void tmem_ld_frag<2>(uint32_t taddr, float (*f)[4]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.16x256b.x2.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i >> 2][i & 3] = __uint_as_float(r[i]);
}

template <>
__device__ __forceinline__ void tmem_ld_frag<4>(uint32_t taddr, float (*f)[4]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x4.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) f[i >> 2][i & 3] = __uint_as_float(r[i]);
}

// any even number of groups, as loads of 4 and 2 groups (8 columns each)
template <int NF>
__device__ __forceinline__ void tmem_ld_frag(uint32_t taddr, float (*f)[4]) {
  static_assert(NF % 2 == 0 && NF > 4, "even group count");
  tmem_ld_frag<4>(taddr, f);
  tmem_ld_frag<NF - 4>(taddr + 32, f + 4);
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// lane field of a TMEM address: bits [31:16]; column: bits [15:0]
__device__ __forceinline__ uint32_t tmem_addr(uint32_t base, uint32_t lane, uint32_t col) {
  return base + (lane << 16) + col;
}

// ---------------------------------------------------------------------------
// descriptors and the MMA
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

// bf16 x bf16 -> f32, M x N, A/B major (0 = K-major, 1 = MN-major)
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, int a_major, int b_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(a_major) << 15) |
         (static_cast<uint32_t>(b_major) << 16) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]^T, issued by one thread
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// arrive on bar once every MMA this thread issued before has completed
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// byte offset of element (row, col) of a [rows x 64] bf16 SW128 tile
__device__ __forceinline__ uint32_t sw128_off(int row, int col) {
  return static_cast<uint32_t>(row * 128 + ((((col >> 3) ^ (row & 7)) << 4) | ((col & 7) << 1)));
}

}  // namespace tc
}  // namespace gdn2
