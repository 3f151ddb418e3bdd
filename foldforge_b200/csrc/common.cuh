// Device primitives shared by every sm_100a kernel of the Pairformer pair stack.
//
// * mbarrier waits are BOUNDED: after FFB_WAIT_CYCLES of polling (or as soon as another
//   thread has recorded an error) the waiter records a status in the launch's error word
//   and returns false; kernels then skip to their clean-up (TMEM is always freed).
// * TMA: tiled bulk tensor loads / stores (no cluster multicast anywhere in this library).
// * tcgen05: TMEM allocation, kind::f16 MMA (bf16 operands, fp32 accumulators in TMEM),
//   commit to an mbarrier, 32x32b TMEM loads.
// * UMMA descriptors: the shared-memory matrix descriptor and the instruction descriptor,
//   with the field layout of the sm_100 matrix-descriptor format (start address >> 4 at
//   bit 0, leading byte offset >> 4 at bit 16, stride byte offset >> 4 at bit 32,
//   version 1 at bit 46, swizzle mode at bit 61).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#ifndef FFB_WAIT_CYCLES
// ~2 s at 1.9 GHz: far above any legitimate wait, short enough to end a stuck launch.
#define FFB_WAIT_CYCLES (4000000000ll)
#endif

namespace ffb {

// Error codes written to the device error word (first writer wins).
enum DeviceError : int {
  kErrNone = 0,
  kErrTimeoutLoad = 101,   // a TMA load never completed
  kErrTimeoutMma = 102,    // an MMA commit never arrived
  kErrTimeoutEmpty = 103,  // a consumer never released a stage
  kErrTimeoutStore = 104,
  kErrBadLaunch = 105,     // launch geometry the kernel was not written for
  kErrTimeoutPeer = 106,   // another rank never signalled an exchange
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void set_error(int* err, int code) {
  if (err != nullptr) atomicCAS(err, 0, code);
}

__device__ __forceinline__ bool error_raised(const int* err) {
  return err != nullptr && *reinterpret_cast<const volatile int*>(err) != 0;
}

// ------------------------------------------------------------------ mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: a thread whose phase is not complete is suspended by
// the hardware until the phase completes or `ns` nanoseconds pass, instead of polling.
__device__ __forceinline__ bool mbar_try_wait_suspend(uint32_t bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete. Returns false (and records
// `code`) after FFB_WAIT_CYCLES, or when another thread has already recorded an error
// (checked about every million cycles, so the wait loop issues almost nothing and reads
// no global memory while it waits).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  const long long start = clock64();
  long long checked = start;
  while (true) {
    if (mbar_try_wait_suspend(a, parity, 20000u)) return true;
    const long long now = clock64();
    if (now - checked > (1ll << 20)) {
      checked = now;
      if (error_raised(err)) return false;
      if (now - start > FFB_WAIT_CYCLES) {
        set_error(err, code);
        return false;
      }
    }
  }
}

// ------------------------------------------------------------------ fences / barriers
// Generic-proxy writes to shared memory made visible to the async proxy (TMA store,
// tcgen05.mma operand reads).
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void named_barrier(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Named barrier that also ORs a predicate over the participating threads: every thread
// gets the same answer, so a group can leave a loop together.
__device__ __forceinline__ bool named_barrier_or(int id, int threads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}\n"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred)), "r"(id), "r"(threads)
      : "memory");
  return r != 0;
}

// ------------------------------------------------------------------ TMA
__device__ __forceinline__ void tma_prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z,
                                            int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}

__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
               : "memory");
}

__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int x, int y, int z, int w) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z), "r"(w)
               : "memory");
}

__device__ __forceinline__ void tma_store_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Wait until the committed stores have finished READING shared memory.
__device__ __forceinline__ void tma_store_wait_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

__device__ __forceinline__ void tma_store_wait_all0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Wait until every committed store group but the most recent one has finished READING
// shared memory (two staging buffers used in turn).
__device__ __forceinline__ void tma_store_wait_read1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}

// Plain (untiled) bulk copy global -> shared; addresses 16-byte aligned, size % 16 == 0.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ------------------------------------------------------------------ tcgen05 / TMEM
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, one instruction of shape (M, N, 16).
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when every tcgen05.mma issued so far by this thread completes.
// The same with the A operand in TMEM (M rows on the 128 lanes, K along the columns, two
// 16-bit elements per 32-bit column, so 16 K elements = 8 columns).
__device__ __forceinline__ void mma_bf16_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 bits, 16 consecutive columns: thread t of the warp receives lane
// (warp % 4) * 32 + t, columns [col, col + 16).
// TMEM stores (32 lanes x N columns per warp, lane = thread); tmem_st_wait before the
// stored values may be read by another thread or the tensor core.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st1(uint32_t taddr, uint32_t r) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(taddr), "r"(r) : "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld1(uint32_t taddr, uint32_t& r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr) : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
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

// ------------------------------------------------------------------ UMMA descriptors
// K-major operand tile in the 128-byte swizzle layout: rows of 64 bf16 (128 B), 8-row
// groups 1024 B apart (stride byte offset), tile base 1024-byte aligned. Advancing K by
// 16 elements inside the 128-byte row is +32 bytes on the start address.
__device__ __forceinline__ uint64_t desc_kmajor_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;               // leading byte offset (unused for swizzled K-major)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;       // stride byte offset: 8 rows x 128 B
  d |= static_cast<uint64_t>(1u) << 46;               // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2u) << 61;               // SWIZZLE_128B
  return d;
}

// K-major operand tile in the 64-byte swizzle layout: rows of 32 bf16 (64 B), 8-row groups
// 512 B apart; +32 bytes on the start address advances K by 16 elements.
__device__ __forceinline__ uint64_t desc_kmajor_sw64(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>(512u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(4u) << 61;  // SWIZZLE_64B
  return d;
}

// MN-major operand in the 128-byte swizzle layout: each 128-byte row holds 64 consecutive
// M (or N) elements of one K index, 8-row K groups `sbo` bytes apart (1024 for a dense
// tile), and the next 64-element M/N block `lbo` bytes further. Advancing K by 16 is
// +16 rows (2 K groups) on the start address.
__device__ __forceinline__ uint64_t desc_mnmajor_sw128(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor: bf16 A (K-major) x bf16 B (MN-major) -> fp32, shape M x N.
__host__ __device__ constexpr uint32_t idesc_bf16_f32_bmn(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16)  // B is MN-major
         | (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

// Instruction descriptor: bf16 A (MN-major) x bf16 B (K-major) -> fp32, shape M x N.
__host__ __device__ constexpr uint32_t idesc_bf16_f32_amn(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (1u << 15)  // A is MN-major
         | (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

// Instruction descriptor: bf16 x bf16 -> fp32, both operands K-major, shape M x N.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int m, int n) {
  return (1u << 4)                                  // D format: f32
         | (1u << 7)                                // A format: bf16
         | (1u << 10)                               // B format: bf16
         | (static_cast<uint32_t>(n >> 3) << 17)    // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);   // M / 16
}

// Instruction descriptor: f16 x f16 -> fp32, both operands K-major, shape M x N.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int m, int n) {
  return (1u << 4)                                  // D format: f32
         | (static_cast<uint32_t>(n >> 3) << 17)    // A, B format: f16 (0)
         | (static_cast<uint32_t>(m >> 4) << 24);
}

// Byte offset of element (row, col) (col in bf16 units, < 64) inside a K-major SW128 atom
// column whose rows are 128 bytes: the 16-byte chunk index is XOR-ed with (row % 8).
__device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t col) {
  const uint32_t chunk = (col >> 3) ^ (row & 7u);
  return row * 128u + chunk * 16u + (col & 7u) * 2u;
}

// Byte offset of element (row, col) (col in bf16 units, < 32) inside a K-major SW64 tile
// whose rows are 64 bytes (tile base 512-byte aligned): the 16-byte chunk index is XOR-ed
// with (row / 2) % 4, the 64-byte swizzle pattern of TMA and the UMMA descriptor.
__device__ __forceinline__ uint32_t sw64_offset(uint32_t row, uint32_t col) {
  const uint32_t chunk = ((col >> 3) ^ (row >> 1)) & 3u;
  return row * 64u + chunk * 16u + (col & 7u) * 2u;
}

// ------------------------------------------------------------------ math helpers
__device__ __forceinline__ float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }

// LayerNorm statistics (mean, 1/sqrt(var + 1e-5)) of row `row` of a K-major SW128 tile of
// 128 bf16 channels stored as two 64-channel blocks `block_bytes` apart: one pass on the
// paired fp32 pipe over the row held in registers, summing x - x0 and its square (shifted by
// the row's first channel, so the variance does not cancel when |mean| >> std).
__device__ __forceinline__ void ln_stats_c128(const uint8_t* tile, int block_bytes, int row, float& mean,
                                              float& rstd) {
  uint4 v[16];
#pragma unroll
  for (int kb = 0; kb < 2; ++kb)
#pragma unroll
    for (int q = 0; q < 8; ++q)
      v[kb * 8 + q] = *reinterpret_cast<const uint4*>(tile + kb * block_bytes + sw128_offset(row, q * 8));
  const float x0 = bf16_lo(v[0].x);
  uint64_t shift, s1 = 0, s2 = 0;
  asm("mov.b64 %0, {%1, %1};" : "=l"(shift) : "f"(-x0));
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint64_t x, d;
      asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "f"(bf16_lo(w[j])), "f"(bf16_hi(w[j])));
      asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(x), "l"(shift));
      asm("add.rn.f32x2 %0, %1, %2;" : "=l"(s1) : "l"(s1), "l"(d));
      asm("fma.rn.f32x2 %0, %1, %1, %2;" : "=l"(s2) : "l"(d), "l"(s2));
    }
  }
  float a1, b1, a2, b2;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a1), "=f"(b1) : "l"(s1));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a2), "=f"(b2) : "l"(s2));
  const float dm = (a1 + b1) * (1.0f / 128.0f);
  mean = x0 + dm;
  rstd = rsqrtf(fmaxf((a2 + b2) * (1.0f / 128.0f) - dm * dm, 0.f) + 1e-5f);
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + __expf(-x)); }

// Hardware tanh approximation (one MUFU op; max relative error about 2^-11), enough for
// values that are rounded to bf16 next.
__device__ __forceinline__ float tanh_fast(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// sigmoid(x) = 0.5 tanh(x / 2) + 0.5: one MUFU op and two FMAs.
__device__ __forceinline__ float sigmoid_fast(float x) { return fmaf(0.5f, tanh_fast(0.5f * x), 0.5f); }

// ---- paired fp32 arithmetic (sm_100 f32x2) and f16x2 helpers
__device__ __forceinline__ uint64_t f32x2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f32x2_split(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t add_f32x2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t mul_f32x2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fma_f32x2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
// {lo, hi} fp32 -> f16x2 (lo in the low half)
__device__ __forceinline__ uint32_t f16x2_from(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint32_t ex2_f16x2(uint32_t x) {
  uint32_t r;
  asm("ex2.approx.f16x2 %0, %1;" : "=r"(r) : "r"(x));
  return r;
}
__device__ __forceinline__ uint32_t add_f16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ float f16x2_sum(uint32_t v) {
  __half2 h = *reinterpret_cast<__half2*>(&v);
  return __low2float(h) + __high2float(h);
}

// 2^d for a pair of fp32 values on the FMA and integer pipes (no MUFU): d is clamped to
// [-126, 0], split as n + f with n = round(d) (the 1.5 * 2^23 rounding constant) and
// f in [-0.5, 0.5]; 2^f is a cubic fitted to relative error (max 7.8e-5 on the interval)
// and 2^n enters as an integer add to the exponent field. Inputs below -126 (masked
// logits, -inf) give at most 2^-126.
__device__ __forceinline__ void exp2_poly_x2(uint64_t d, float& e0, float& e1) {
  float d0, d1;
  f32x2_split(d, d0, d1);
  const uint64_t dc = f32x2(fmaxf(d0, -126.0f), fmaxf(d1, -126.0f));
  const uint64_t t = add_f32x2(dc, f32x2(12582912.0f, 12582912.0f));
  const uint64_t n = add_f32x2(t, f32x2(-12582912.0f, -12582912.0f));
  const uint64_t fr = fma_f32x2(n, f32x2(-1.0f, -1.0f), dc);
  uint64_t p = fma_f32x2(f32x2(0.05508876592f, 0.05508876592f), fr, f32x2(0.24260465801f, 0.24260465801f));
  p = fma_f32x2(p, fr, f32x2(0.69327628613f, 0.69327628613f));
  p = fma_f32x2(p, fr, f32x2(0.99992889166f, 0.99992889166f));
  float p0, p1, t0, t1;
  f32x2_split(p, p0, p1);
  f32x2_split(t, t0, t1);
  e0 = __uint_as_float(__float_as_uint(p0) + (__float_as_uint(t0) << 23));
  e1 = __uint_as_float(__float_as_uint(p1) + (__float_as_uint(t1) << 23));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

}  // namespace ffb
