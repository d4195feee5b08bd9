// Shared device infrastructure of the kdn_b200 library (sm_100a).
//
// * Warp-level matrix products on mma.sync.m16n8k16 (bf16 operands, fp32
//   accumulators) with operands staged in shared memory and fetched by
//   ldmatrix, plus an fp32 SIMT twin with the identical accumulator layout
//   (the fp32 "debug" precision of the library).
// * cp.async row copies from HBM into shared memory.
// * Host-side error state for the C ABI.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "../../../include/kdn_b200.h"

namespace kdn {

using bf16 = __nv_bfloat16;

// ---------------------------------------------------------------------------
// Host error state (kdn_api.cu)
// ---------------------------------------------------------------------------
int set_error(int code, const char* fmt, ...);
int check_launch(const char* what);

// ---------------------------------------------------------------------------
// Scalar helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(bf16 x) { return __bfloat162float(x); }
template <class T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ bf16 from_f<bf16>(float x) { return __float2bfloat16_rn(x); }

__device__ __forceinline__ float ex2(float x) { return exp2f(x); }
// Hardware base-2 exponential (MUFU ex2, flushes subnormal results to zero).
__device__ __forceinline__ float ex2a(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Lane l ends with the warp sum of v[l % N] (N = 8, 16 or 32): a butterfly
// that halves the values exchanged at every step.
template <int N>
__device__ __forceinline__ float transpose_reduce(float (&v)[N]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int off = N / 2; off >= 1; off >>= 1) {
    const bool upper = lane & off;
#pragma unroll
    for (int i = 0; i < off; ++i) {
      const float send = upper ? v[i] : v[i + off];
      const float keep = upper ? v[i + off] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  float s = v[0];
#pragma unroll
  for (int o = N; o < 32; o <<= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  return s;
}

// Sum of v[j] over all K threads of the block for each of N tokens; result in
// out[j] (shared) after the second barrier.
template <int K, int N>
__device__ __forceinline__ void block_token_sums(float (&v)[N], float* red /* [K/32][N] */, float* out /* [N] */) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float s = transpose_reduce<N>(v);
  if (lane < N) red[warp * N + lane] = s;
  __syncthreads();
  if (threadIdx.x < N) {
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < K / 32; ++w) acc += red[w * N + threadIdx.x];
    out[threadIdx.x] = acc;
  }
  __syncthreads();
}

// Store two adjacent values (one 32-bit store for bf16, one 64-bit for fp32).
__device__ __forceinline__ void st_pair(bf16* p, float a, float b) {
  *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(a, b);
}
__device__ __forceinline__ void st_pair(float* p, float a, float b) { *reinterpret_cast<float2*>(p) = make_float2(a, b); }

// 8 consecutive values as fp32 (16-byte aligned source).
__device__ __forceinline__ void ld8(float (&d)[8], const bf16* p) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    d[2 * i] = f.x;
    d[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void ld8(float (&d)[8], const float* p) {
  const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
  d[0] = a.x; d[1] = a.y; d[2] = a.z; d[3] = a.w; d[4] = b.x; d[5] = b.y; d[6] = b.z; d[7] = b.w;
}
__device__ __forceinline__ void st8(bf16* p, const float (&s)[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(s[2 * i], s[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}
__device__ __forceinline__ void st8(float* p, const float (&s)[8]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(s[0], s[1], s[2], s[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(s[4], s[5], s[6], s[7]);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---------------------------------------------------------------------------
// Tensor-core fragments (mma.sync.m16n8k16, row.col, bf16 x bf16 -> fp32).
// Accumulator layout per lane (g = lane/4, t = lane%4): c0,c1 at row g,
// cols 2t,2t+1; c2,c3 at row g+8, same cols.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ void ldsm_x2(uint32_t (&r)[2], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];\n"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t (&r)[2], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];\n"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <int MT, int NT>
__device__ __forceinline__ void zero_acc(float (&acc)[MT][NT][4]) {
#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.f;
}

// Warp product acc[MT][NT] += A[m0 : m0+16MT, k0:k1] * B[k0:k1, n0 : n0+8NT].
//   AK: A(m,k) = A[m*lda + k] (k contiguous), else A(m,k) = A[k*lda + m].
//   BK: B(k,n) = B[n*ldb + k] (k contiguous), else B(k,n) = B[k*ldb + n].
// k0, k1 multiples of 16.  bf16 operands live in shared memory with 16-byte
// aligned rows.
template <int MT, int NT, bool AK, bool BK>
__device__ __forceinline__ void wgemm(float (&acc)[MT][NT][4], const bf16* A, int lda, const bf16* B, int ldb,
                                      int m0, int n0, int k0, int k1) {
  const int lane = threadIdx.x & 31;
  const int mi = lane >> 3, r = lane & 7;
  for (int k = k0; k < k1; k += 16) {
    uint32_t a[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      if constexpr (AK) {
        ldsm_x4(a[mt], A + (size_t)(m0 + mt * 16 + (lane & 15)) * lda + k + (lane >> 4) * 8);
      } else {
        ldsm_x4_t(a[mt], A + (size_t)(k + (mi >> 1) * 8 + r) * lda + m0 + mt * 16 + (mi & 1) * 8);
      }
    }
#pragma unroll
    for (int nt = 0; nt + 1 < NT; nt += 2) {
      uint32_t b[4];
      if constexpr (BK) {
        ldsm_x4(b, B + (size_t)(n0 + nt * 8 + (mi >> 1) * 8 + r) * ldb + k + (mi & 1) * 8);
      } else {
        ldsm_x4_t(b, B + (size_t)(k + (mi & 1) * 8 + r) * ldb + n0 + nt * 8 + (mi >> 1) * 8);
      }
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        mma_16816(acc[mt][nt], a[mt], b[0], b[1]);
        mma_16816(acc[mt][nt + 1], a[mt], b[2], b[3]);
      }
    }
    if constexpr (NT % 2 == 1) {
      constexpr int nt = NT - 1;
      const int l = lane & 15, mj = l >> 3, rr = l & 7;
      uint32_t b[2];
      if constexpr (BK) {
        ldsm_x2(b, B + (size_t)(n0 + nt * 8 + rr) * ldb + k + mj * 8);
      } else {
        ldsm_x2_t(b, B + (size_t)(k + mj * 8 + rr) * ldb + n0 + nt * 8);
      }
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) mma_16816(acc[mt][nt], a[mt], b[0], b[1]);
    }
  }
}

// fp32 SIMT twin of wgemm: same accumulator layout, operands anywhere.
template <int MT, int NT, bool AK, bool BK>
__device__ __forceinline__ void wgemm(float (&acc)[MT][NT][4], const float* A, int lda, const float* B, int ldb,
                                      int m0, int n0, int k0, int k1) {
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  for (int k = k0; k < k1; ++k) {
    float alo[MT], ahi[MT];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const int m = m0 + mt * 16 + g;
      if constexpr (AK) {
        alo[mt] = A[(size_t)m * lda + k];
        ahi[mt] = A[(size_t)(m + 8) * lda + k];
      } else {
        alo[mt] = A[(size_t)k * lda + m];
        ahi[mt] = A[(size_t)k * lda + m + 8];
      }
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int n = n0 + nt * 8 + 2 * t;
      float b0, b1;
      if constexpr (BK) {
        b0 = B[(size_t)n * ldb + k];
        b1 = B[(size_t)(n + 1) * ldb + k];
      } else {
        b0 = B[(size_t)k * ldb + n];
        b1 = B[(size_t)k * ldb + n + 1];
      }
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        acc[mt][nt][0] = fmaf(alo[mt], b0, acc[mt][nt][0]);
        acc[mt][nt][1] = fmaf(alo[mt], b1, acc[mt][nt][1]);
        acc[mt][nt][2] = fmaf(ahi[mt], b0, acc[mt][nt][2]);
        acc[mt][nt][3] = fmaf(ahi[mt], b1, acc[mt][nt][3]);
      }
    }
  }
}

// Visit the (row, col) coordinates a lane holds in an accumulator tile.
// f(mt, nt, e, row, col) for every element.
template <int MT, int NT, class F>
__device__ __forceinline__ void for_acc(int m0, int n0, F&& f) {
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) f(mt, nt, e, m0 + mt * 16 + g + (e >> 1) * 8, n0 + nt * 8 + 2 * t + (e & 1));
}

// Store an accumulator tile to a row-major buffer (ld elements), converting;
// adjacent column pairs go out as one store.
template <class T, int MT, int NT>
__device__ __forceinline__ void store_acc(T* dst, int ld, const float (&acc)[MT][NT][4], int m0, int n0) {
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = m0 + mt * 16 + g + 8 * h, col = n0 + nt * 8 + 2 * t;
        st_pair(dst + (size_t)row * ld + col, acc[mt][nt][2 * h], acc[mt][nt][2 * h + 1]);
      }
}

// Visit accumulator element pairs (adjacent columns): f(mt, nt, h, row, col, v0, v1).
template <int MT, int NT, class F>
__device__ __forceinline__ void for_acc_pairs(const float (&acc)[MT][NT][4], int m0, int n0, F&& f) {
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int h = 0; h < 2; ++h)
        f(mt, nt, h, m0 + mt * 16 + g + 8 * h, n0 + nt * 8 + 2 * t, acc[mt][nt][2 * h], acc[mt][nt][2 * h + 1]);
}

// Two A tiles from different buffers sharing the B fragments:
// acc[i] += A_i[m0 : m0+16, k] * B[k, n0 : n0+8NT].
template <int NT, bool AK, bool BK>
__device__ __forceinline__ void wgemm_dual(float (&acc)[2][NT][4], const bf16* A0, const bf16* A1, int lda,
                                           const bf16* B, int ldb, int m0, int n0, int k0, int k1) {
  static_assert(NT % 2 == 0 && AK, "dual-A product: row-major A, even NT");
  const int lane = threadIdx.x & 31;
  const int mi = lane >> 3, r = lane & 7;
  for (int k = k0; k < k1; k += 16) {
    uint32_t a[2][4];
    ldsm_x4(a[0], A0 + (size_t)(m0 + (lane & 15)) * lda + k + (lane >> 4) * 8);
    ldsm_x4(a[1], A1 + (size_t)(m0 + (lane & 15)) * lda + k + (lane >> 4) * 8);
#pragma unroll
    for (int nt = 0; nt < NT; nt += 2) {
      uint32_t b[4];
      if constexpr (BK) {
        ldsm_x4(b, B + (size_t)(n0 + nt * 8 + (mi >> 1) * 8 + r) * ldb + k + (mi & 1) * 8);
      } else {
        ldsm_x4_t(b, B + (size_t)(k + (mi & 1) * 8 + r) * ldb + n0 + nt * 8 + (mi >> 1) * 8);
      }
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        mma_16816(acc[i][nt], a[i], b[0], b[1]);
        mma_16816(acc[i][nt + 1], a[i], b[2], b[3]);
      }
    }
  }
}
template <int NT, bool AK, bool BK>
__device__ __forceinline__ void wgemm_dual(float (&acc)[2][NT][4], const float* A0, const float* A1, int lda,
                                           const float* B, int ldb, int m0, int n0, int k0, int k1) {
  float a0[1][NT][4], a1[1][NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      a0[0][nt][e] = acc[0][nt][e];
      a1[0][nt][e] = acc[1][nt][e];
    }
  wgemm<1, NT, AK, BK>(a0, A0, lda, B, ldb, m0, n0, k0, k1);
  wgemm<1, NT, AK, BK>(a1, A1, lda, B, ldb, m0, n0, k0, k1);
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      acc[0][nt][e] = a0[0][nt][e];
      acc[1][nt][e] = a1[0][nt][e];
    }
}

// ---------------------------------------------------------------------------
// Asynchronous copies HBM -> shared (16-byte granules, L2-only caching).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(smem)), "l"(gmem));
}
// 4- and 8-byte copies (L1-allocating; the only sizes below 16 bytes cp.async takes)
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(smem_u32(smem)), "l"(gmem));
}
__device__ __forceinline__ void cp_async8(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(smem_u32(smem)), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::); }
// All but the newest N committed cp.async groups have landed.
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// Copy `rows` rows of `row_bytes` (multiple of 16) from a strided global
// source into a padded destination.  Rows >= valid are zero-filled.  `smem`
// selects cp.async (shared destination) or plain copies (global destination,
// fp32 debug precision).
template <bool SMEM>
__device__ __forceinline__ void copy_rows(void* dst, size_t dst_stride, const void* src, size_t src_stride,
                                          int rows, int valid, int row_bytes) {
  const int per_row = row_bytes / 16;
  const int total = rows * per_row;
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const int row = i / per_row, col = i - row * per_row;
    char* d = static_cast<char*>(dst) + row * dst_stride + col * 16;
    if (row < valid) {
      const char* s = static_cast<const char*>(src) + row * src_stride + col * 16;
      if constexpr (SMEM) {
        cp_async16(d, s);
      } else {
        *reinterpret_cast<int4*>(d) = *reinterpret_cast<const int4*>(s);
      }
    } else {
      *reinterpret_cast<int4*>(d) = make_int4(0, 0, 0, 0);
    }
  }
}

__host__ __device__ constexpr size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// ---------------------------------------------------------------------------
// Packed variable-length batches.  N sequences lie back to back along T of a
// B = 1 batch; each is cut into its own 64-token chunks (the last one
// partial), numbered globally in packed order.  The table (kdn_varlen_plan)
// is one int32 array: tok[N+1] token offsets (cu_seqlens), chunk[N+1] first
// global chunk of each sequence, order[N] the sequences longest first (the
// stream slots of the sequential passes, so that the longest chains start
// first), seq[NC] the sequence of each global chunk.  n = 0: a fixed-length
// batch (no table).
// ---------------------------------------------------------------------------
constexpr int kVarlenChunk = 64;
struct Varlen {
  const int* tok;
  const int* chunk;
  const int* order;
  const int* seq;
  int n;
  __host__ __device__ bool on() const { return n > 0; }
};
inline Varlen varlen_view(const int32_t* table, int64_t n) {
  Varlen v{nullptr, nullptr, nullptr, nullptr, 0};
  if (table && n > 0) {
    v.tok = table;
    v.chunk = table + (n + 1);
    v.order = table + 2 * (n + 1);
    v.seq = table + 2 * (n + 1) + n;
    v.n = (int)n;
  }
  return v;
}
// First token (packed index) and length of global chunk gc, and its sequence.
__device__ __forceinline__ void varlen_span(const Varlen& v, int gc, int& t0, int& len, int& s) {
  s = v.seq[gc];
  t0 = v.tok[s] + (gc - v.chunk[s]) * kVarlenChunk;
  len = min(kVarlenChunk, v.tok[s + 1] - t0);
}

// ---------------------------------------------------------------------------
// Bulk copies (TMA) and mbarriers.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory"); }
// Generic-proxy shared-memory writes become visible to bulk (async-proxy) reads.
__device__ __forceinline__ void fence_async_shared() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}
// Barrier `id` (1..15) among `n` threads (a multiple of 32), leaving the
// other warps of the block free.
__device__ __forceinline__ void bar_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(n) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Status word bits (the first int of the call's status header).
constexpr int kStatusGaveUp = 1;     // a wait ran out of polls: the call's results are invalid
constexpr int kStatusSlowWait = 2;   // a wait needed more polls than the debug limit (results valid)
constexpr int kWaitPolls = 1 << 20;  // hard poll limit of every mbarrier wait

// Non-blocking probe of phase `parity` (try_wait may suspend the thread for a
// while before it reports failure; test_wait never does).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Wait for phase `parity` of an mbarrier: one non-blocking probe, then at
// most kWaitPolls polls; on time-out set kStatusGaveUp in *status (when
// given) and return so the kernel cannot hang.  status[1] is a debug poll
// limit written by the host before the launch (0 = off): a wait that needs
// that many polls or more (the probe counts as the first) sets
// kStatusSlowWait and keeps waiting up to the hard limit, so the host's
// status check can be exercised without any copy left in flight.
__device__ __forceinline__ void mbar_wait(uint64_t* bar, unsigned parity, int* status) {
  if (mbar_test_wait(bar, parity)) return;
  const int soft = status ? *reinterpret_cast<volatile int*>(status + 1) : 0;
  for (int i = 1; i <= kWaitPolls; ++i) {
    if (soft > 0 && i == soft) atomicOr(status, kStatusSlowWait);
    if (mbar_try_wait(bar, parity)) return;
  }
  if (status) atomicOr(status, kStatusGaveUp);
}

// 4-D tiled tensor load (box given by the tensor map) into shared memory.
__device__ __forceinline__ void tma_load_4d(void* dst, const void* tmap, int c0, int c1, int c2, int c3,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];\n" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}
// Contiguous global -> shared copy (16-byte aligned, size multiple of 16).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
// Contiguous shared -> global copy, tracked by this thread's bulk group.
__device__ __forceinline__ void bulk_s2g(void* dst, const void* src, unsigned bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;\n" ::"l"(dst), "r"(smem_u32(src)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;\n" ::: "memory"); }
// This thread's committed bulk stores, all but the newest N groups, have
// finished reading shared memory.
template <int N = 0>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;\n" ::"n"(N) : "memory");
}
// ... and finished writing global memory.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory"); }

}  // namespace kdn
