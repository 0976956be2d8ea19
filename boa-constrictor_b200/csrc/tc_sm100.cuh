// sm_100a building blocks: mbarriers with bounded waits, bulk async copies,
// TMEM allocation / load / store, tcgen05.mma and its descriptors.
//
// Operand layout used everywhere in this library ("SW128 K-major"):
//   a tile is R rows x 128 bytes of K (32 tf32 / 64 fp16|bf16 elements);
//   row r lives at byte r*128, and its 16-byte chunk c is stored at chunk
//   position c ^ (r % 8) (the 128-byte swizzle).  Eight rows (1024 bytes) form
//   one swizzle atom, so the stride between 8-row groups (SBO) is 1024 bytes.
//   Tile bases are 1024-byte aligned; advancing K by one MMA step (32 bytes)
//   inside a tile adds 32 bytes to the descriptor start address.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

namespace boa {
namespace tc {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ----------------------------- mbarrier ------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait.  Gives up (returns false) when another thread raised *abort
// or when `budget` SM clock cycles pass; in the latter case it raises *abort.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          long long budget) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > budget) {
      *abort_flag = 1;
      return false;
    }
  }
}

// --------------------------- bulk async copy --------------------------------
// Untiled bulk copy global -> this CTA's shared memory, completion counted in
// bytes on `bar`.  Addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
// Bulk prefetch of [src, src+bytes) into L2 (16-byte aligned, multiple of 16).
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Per-warpgroup register budget (all four warps of a warpgroup execute the
// same instruction); an increase waits until other warpgroups' decreases have
// returned the registers to the block's launch allocation.
template <int N>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

// Make this thread's generic-proxy shared-memory writes visible to the async
// proxy (tensor core operand reads).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// --------------------------------- TMEM -------------------------------------
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
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 lanes x 16 consecutive 32-bit columns: thread i of the warp receives lane
// (taddr.lane + i), columns taddr.col .. taddr.col+15.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, float (&v)[4]) {
  uint32_t r[4];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(r[i]);
}
// Two 8-column loads (32 lanes each) at a0 and a1, summed: the hi and lo
// accumulators of eight value columns of a split-kind GEMM.
__device__ __forceinline__ void tmem_ld8_sum(uint32_t a0, uint32_t a1, float (&v)[8]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%16];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%8,%9,%10,%11,%12,%13,%14,%15}, [%17];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(a0), "r"(a1)
      : "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]) + __uint_as_float(r[8 + i]);
}
__device__ __forceinline__ void tmem_ld4_sum(uint32_t a0, uint32_t a1, float (&v)[4]) {
  uint32_t r[8];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%8];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x4.b32 {%4,%5,%6,%7}, [%9];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
      : "r"(a0), "r"(a1)
      : "memory");
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(r[i]) + __uint_as_float(r[4 + i]);
}

// As tmem_ld8_sum / tmem_ld4_sum, with the second load scaled: a0 + 2^-11 a1
// (one fma, a single rounding), for the kind-4 accumulators.
__device__ __forceinline__ void tmem_ld8_sum_s11(uint32_t a0, uint32_t a1, float (&v)[8]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%16];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%8,%9,%10,%11,%12,%13,%14,%15}, [%17];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(a0), "r"(a1)
      : "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __fmaf_rn(__uint_as_float(r[8 + i]), 0x1p-11f, __uint_as_float(r[i]));
}
__device__ __forceinline__ void tmem_ld4_sum_s11(uint32_t a0, uint32_t a1, float (&v)[4]) {
  uint32_t r[8];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%8];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x4.b32 {%4,%5,%6,%7}, [%9];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
      : "r"(a0), "r"(a1)
      : "memory");
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = __fmaf_rn(__uint_as_float(r[4 + i]), 0x1p-11f, __uint_as_float(r[i]));
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15]))
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 32 lanes x 8 columns store; completion is awaited with tmem_wait_st().
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const float (&v)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr),
               "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
               "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
               "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7]))
               : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ------------------------------ tcgen05.mma ---------------------------------
// Shared-memory matrix descriptor for a SW128 K-major operand (see top).
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);   // bits 0-13: start address >> 4
  d |= (uint64_t)1 << 16;                       // bits 16-29: leading byte offset (unused for SW128 K-major)
  d |= (uint64_t)(1024 >> 4) << 32;             // bits 32-45: stride byte offset = 1024 B
  d |= (uint64_t)1 << 46;                       // bits 46-47: descriptor version 1 (sm_100)
  d |= (uint64_t)2 << 61;                       // bits 61-63: 128-byte swizzle
  return d;
}

// Operand kinds (the BOA_WEIGHTS_* values): 0 = tf32 (fp32 storage), 1 = bf16,
// 2 = fp16, 3 = 3xTF32.  kHiLo = 2 marks the split kind: every fp32 value v is
// stored as two tf32 halves, hi = rna_tf32(v) and lo = rna_tf32(v - hi).  The
// activation operand B carries the halves as separate rows (hi of value column
// n in row n, lo in row n + CT/2, so one MMA with N = CT multiplies a weight
// tile by both), and every weight tile is followed by the tile of its lo
// halves.  An accumulator column n < CT/2 then sums A_hi*B_hi + A_lo*B_hi and
// column n + CT/2 sums A_hi*B_lo + A_lo*B_lo; their fp32 sum is the product
// (A_hi + A_lo)(B_hi + B_lo), i.e. each operand carries 22 significant bits
// instead of tf32's 11 (the 3xTF32 scheme, with the A_lo*B_lo term kept
// because it rides in the same instructions).
template <int KIND>
struct OpKind;
template <>
struct OpKind<0> {
  static constexpr int kElemBytes = 4;
  static constexpr uint32_t kFmt = 2;  // TF32
  static constexpr int kHiLo = 1;
};
template <>
struct OpKind<1> {
  static constexpr int kElemBytes = 2;
  static constexpr uint32_t kFmt = 1;  // BF16
  static constexpr int kHiLo = 1;
};
template <>
struct OpKind<2> {
  static constexpr int kElemBytes = 2;
  static constexpr uint32_t kFmt = 0;  // F16
  static constexpr int kHiLo = 1;
};
template <>
struct OpKind<3> {
  static constexpr int kElemBytes = 4;
  static constexpr uint32_t kFmt = 2;  // TF32 (hi and lo halves)
  static constexpr int kHiLo = 2;
};
// Kind 4 = 2xFP16 with a scaled residual (the error-corrected fp16 scheme of
// Ootomo & Yokota, IJHPCA 2022): v = hi + 2^-11 lo', hi = rn_f16(v),
// lo' = rn_f16((v - hi) * 2^11), 22 significant bits for |v| in [2^-14, 65504)
// (below that the absolute error stays under 2^-35).  kHiLo = 4 operand rows
// per value: hi in row n, lo' in row n + VC, hi again in row n + 2 VC and a
// zero row at n + 3 VC (VC = CT / 4).  Every (M tile, K slice) streams the
// weights' hi tile, then their lo' tile: the hi tile multiplies rows
// [0, 2 VC) into accumulator columns [0, 2 VC) and the lo' tile multiplies
// rows [2 VC, 4 VC) into columns [VC, 3 VC), so column n sums W_hi x_hi and
// column n + VC sums W_hi x_lo' + W_lo' x_hi (scale 2^11); the value is
// acc[n] + 2^-11 acc[n + VC] (columns [2 VC, 3 VC) hold W_lo' * 0 and are
// never read).  Half the weight bytes and MMAs of kind 3.
template <>
struct OpKind<4> {
  static constexpr int kElemBytes = 2;
  static constexpr uint32_t kFmt = 0;  // F16 (hi and scaled lo' halves)
  static constexpr int kHiLo = 4;
};

// Instruction descriptor: D fp32, A/B K-major, no negation/sparsity.
template <int KIND>
__host__ __device__ constexpr uint32_t idesc(int M, int N) {
  return (1u << 4) | (OpKind<KIND>::kFmt << 7) | (OpKind<KIND>::kFmt << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

template <int KIND>
__device__ __forceinline__ void mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t id, uint32_t acc) {
  if constexpr (OpKind<KIND>::kFmt == 2) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(id), "r"(acc)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(id), "r"(acc)
        : "memory");
  }
}

// Arrive on `bar` once all previously issued tcgen05.mma of this thread finish.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// ------------------------- operand element stores ---------------------------
// Byte offset of element (row, k) inside a SW128 K-major buffer whose K-slices
// (128 bytes of K each) are `rows` rows tall and stored back to back.
template <int KIND>
__device__ __forceinline__ uint32_t sw128_offset(int row, int k, int rows) {
  constexpr int EB = OpKind<KIND>::kElemBytes;
  constexpr int PER = 128 / EB;                 // elements per 128-byte slice
  const int slice = k / PER;
  const int byte = (k % PER) * EB;
  const int chunk = byte >> 4;
  return (uint32_t)(slice * rows * 128 + row * 128 + (((chunk ^ (row & 7)) << 4) | (byte & 15)));
}

__device__ __forceinline__ uint32_t rna_tf32(float v) {
  uint32_t t;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(t) : "f"(v));
  return t;
}

// Store one activation value with the rounding its operand kind needs.  `rows`
// is the buffer's row count per K slice (the MMA N); for the split kind the
// value's hi half goes to `row` and its lo half to `row + rows / 2`.
template <int KIND>
__device__ __forceinline__ void store_operand(uint8_t* buf, int row, int k, int rows, float v) {
  uint8_t* p = buf + sw128_offset<KIND>(row, k, rows);
  if constexpr (KIND == 4) {
    const int vc = rows / 4;
    const __half hi = __float2half_rn(v);
    const __half lo = __float2half_rn((v - __half2float(hi)) * 2048.0f);
    *reinterpret_cast<unsigned short*>(p) = __half_as_ushort(hi);
    *reinterpret_cast<unsigned short*>(buf + sw128_offset<KIND>(row + vc, k, rows)) = __half_as_ushort(lo);
    *reinterpret_cast<unsigned short*>(buf + sw128_offset<KIND>(row + 2 * vc, k, rows)) = __half_as_ushort(hi);
    *reinterpret_cast<unsigned short*>(buf + sw128_offset<KIND>(row + 3 * vc, k, rows)) = 0;
  } else if constexpr (KIND == 3) {
    const uint32_t hi = rna_tf32(v);
    const uint32_t lo = rna_tf32(v - __uint_as_float(hi));
    *reinterpret_cast<uint32_t*>(p) = hi;
    *reinterpret_cast<uint32_t*>(buf + sw128_offset<KIND>(row + rows / 2, k, rows)) = lo;
  } else if constexpr (KIND == 0) {
    uint32_t t;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(t) : "f"(v));
    *reinterpret_cast<uint32_t*>(p) = t;
  } else if constexpr (KIND == 1) {
    *reinterpret_cast<unsigned short*>(p) = __bfloat16_as_ushort(__float2bfloat16_rn(v));
  } else {
    *reinterpret_cast<unsigned short*>(p) = __half_as_ushort(__float2half_rn(v));
  }
}

}  // namespace tc
}  // namespace boa
