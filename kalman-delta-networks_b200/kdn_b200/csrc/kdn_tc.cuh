// Fifth-generation tensor cores (tcgen05) for the sequential scan passes.
//
// Operand tiles live in shared memory as bf16 matrices cut into 64-column
// blocks of 128-byte rows, the 16-byte granules of each row XOR-swizzled by
// (row % 8) inside 1024-byte atoms (the 128-byte swizzle of the TMA engine
// and of the UMMA canonical layouts).  One such tile X[rows][cols] serves as
//   a K-major operand (MMA rows = X rows, reduction over X cols), or
//   an MN-major operand (MMA rows = X cols, reduction over X rows),
// so a matrix and its transpose never need two copies.  Accumulators live in
// tensor memory (TMEM): an M = 128 product writes lane m, columns n.  One
// thread issues the MMAs; tcgen05.commit signals an mbarrier when they finish.
#pragma once

#include "kdn_common.cuh"

namespace kdn {
namespace tc {

// Byte offset of element (row, col) of a swizzled bf16 tile with `rows` rows.
__host__ __device__ constexpr uint32_t sw_off(int row, int col, int rows) {
  return (uint32_t)((col >> 6) * rows * 128 + row * 128 + ((((col & 63) >> 3) ^ (row & 7)) << 4) + (col & 7) * 2);
}

// Shared-memory matrix descriptor, 128-byte swizzle, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}
// K-major use of tile X (rows = MMA rows): k-step ks reduces over cols 16ks..16ks+15.
__device__ __forceinline__ uint64_t desc_k(const void* X, int rows, int ks) {
  return sdesc(smem_u32(X) + (ks >> 2) * rows * 128 + (ks & 3) * 32, 16);
}
// MN-major use of tile X (cols = MMA rows): k-step ks reduces over rows 16ks..16ks+15.
__device__ __forceinline__ uint64_t desc_mn(const void* X, int rows, int ks) {
  return sdesc(smem_u32(X) + ks * 16 * 128, rows * 128);
}
// Instruction descriptor: bf16 x bf16 -> fp32, M x N, operand majors, optional -A.
__host__ __device__ constexpr uint32_t idesc(int M, int N, bool a_mn, bool b_mn, bool a_neg = false) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_neg << 13) | ((uint32_t)a_mn << 15) |
         ((uint32_t)b_mn << 16) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t id, bool accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(id), "r"((uint32_t)accumulate));
}
// Arrive once on `bar` when every MMA this thread issued so far has completed.
__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Warp-wide TMEM allocation of `ncols` columns (a power of two >= 32); the
// base address is written to shared memory at `slot`.
__device__ __forceinline__ void alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
}
__device__ __forceinline__ void dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}

// 16 consecutive fp32 columns of this thread's lane (warp w reads lanes 32(w%4)..).
__device__ __forceinline__ void ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void st16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
      "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
      "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
      : "memory");
}
__device__ __forceinline__ void wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 16 fp32 values as bf16 into two swizzled granules of row `row` starting at column col (multiple of 16).
__device__ __forceinline__ void st_row16(char* X, int rows, int row, int col, const float (&v)[16], float scale) {
  uint4 u[2];
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(u);
#pragma unroll
  for (int i = 0; i < 8; ++i) h[i] = __floats2bfloat162_rn(scale * v[2 * i], scale * v[2 * i + 1]);
  *reinterpret_cast<uint4*>(X + sw_off(row, col, rows)) = u[0];
  *reinterpret_cast<uint4*>(X + sw_off(row, col + 8, rows)) = u[1];
}

// 4-D tensor-map store of a shared-memory tile (tracked by the bulk group).
__device__ __forceinline__ void tma_store_4d(const void* tmap, const void* src, int c0, int c1, int c2, int c3) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%1, %2, %3, %4}], [%5];" ::"l"(tmap),
               "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(src))
               : "memory");
}

}  // namespace tc

// Shared-memory base rounded up to the 1024-byte alignment of swizzled tiles
// (the caller requests 1024 bytes more than it uses).
__device__ __forceinline__ char* align1024(char* p) {
  return p + ((1024u - (smem_u32(p) & 1023u)) & 1023u);
}

}  // namespace kdn
