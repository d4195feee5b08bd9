// q / k normalisation at the diagonal mixer's boundary (_diag_kdn_normalize,
// lit_gpt/kdn_ops/diag_kdn_chunk.py:2162; Function :2045; kernels :194, :235).
//
// Forward, per [K] row x of q and k (K = 64 or 128):
//   norm = sqrt(sum x^2),  d = max(norm, 1e-12) (NaN kept),
//   q_memory = bf16(q / d_q);  k_gain = k / d_k (fp32);  k_memory = bf16(k_gain)
// and the norms are saved for the backward.  The reference fixes every
// rounding step so its bf16 outputs are bit-reproducible: squares and sums
// in round-to-nearest fp32 without contraction, in PyTorch's reduction order
// for a row held by one warp -- lane l owns elements l, l+32, l+64, l+96,
// combines them as ((a0 + a1) + a2) + a3 (rows >= 16 in the call) or
// (a0 + a2) + (a1 + a3) (fewer rows), then the lanes are summed by a
// shuffle-down tree (offsets 1, 2, 4, 8, 16) and lane 0's total is the
// row's.  IEEE division and square root, no reciprocals.  This file follows
// the same order with the same operations, one warp per row.
//
// Backward, per row, with u the cotangent of the normalised row (q: d
// q_memory; k: d k_gain + d k_memory):
//   z_j = -u_j * ((x_j / d) / d),  g = the same ordered sum of z,
//   dx_j = bf16(u_j / d + (norm >= 1e-12 ? g * (x_j / norm) : 0))
// (fp32 inputs keep the fp32 value), with x_j / norm taken as 0 when norm = 0.
#include "kdn_common.cuh"

namespace kdn {
namespace {

constexpr int kNormWarps = 8;

__device__ __forceinline__ float load_f(const void* p, size_t i, bool bf) {
  return bf ? __bfloat162float(static_cast<const bf16*>(p)[i]) : static_cast<const float*>(p)[i];
}

// The row total of four per-lane values (a_j for elements lane + 32 j) in the
// reference's order; every lane returns lane 0's total.
__device__ __forceinline__ float row_sum(float a0, float a1, float a2, float a3, bool small_rows) {
  float v = small_rows ? __fadd_rn(__fadd_rn(a0, a2), __fadd_rn(a1, a3)) : __fadd_rn(__fadd_rn(__fadd_rn(a0, a1), a2), a3);
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, off));
  return __shfl_sync(0xffffffffu, v, 0);
}

__device__ __forceinline__ float denom_of(float norm) { return norm != norm ? norm : fmaxf(norm, 1e-12f); }

template <int K>
__global__ void __launch_bounds__(32 * kNormWarps) diag_norm_fwd_kernel(
    const void* __restrict__ q, const void* __restrict__ k, int in_bf16, bf16* __restrict__ q_memory,
    float* __restrict__ k_gain, bf16* __restrict__ k_memory, float* __restrict__ q_norm,
    float* __restrict__ k_norm, int64_t n_rows) {
  constexpr int NJ = K / 32;
  const bool bf = in_bf16 != 0, small_rows = n_rows < 16;
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * kNormWarps;
  for (int64_t row = (int64_t)blockIdx.x * kNormWarps + (threadIdx.x >> 5); row < n_rows; row += warps) {
    const size_t base = (size_t)row * K + lane;
    float xq[4] = {0.f, 0.f, 0.f, 0.f}, xk[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      xq[j] = load_f(q, base + 32 * j, bf);
      xk[j] = load_f(k, base + 32 * j, bf);
    }
    const float nq = __fsqrt_rn(row_sum(__fmul_rn(xq[0], xq[0]), __fmul_rn(xq[1], xq[1]), __fmul_rn(xq[2], xq[2]),
                                        __fmul_rn(xq[3], xq[3]), small_rows));
    const float nk = __fsqrt_rn(row_sum(__fmul_rn(xk[0], xk[0]), __fmul_rn(xk[1], xk[1]), __fmul_rn(xk[2], xk[2]),
                                        __fmul_rn(xk[3], xk[3]), small_rows));
    const float dq = denom_of(nq), dk = denom_of(nk);
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      q_memory[base + 32 * j] = __float2bfloat16_rn(__fdiv_rn(xq[j], dq));
      const float kg = __fdiv_rn(xk[j], dk);
      k_gain[base + 32 * j] = kg;
      k_memory[base + 32 * j] = __float2bfloat16_rn(kg);
    }
    if (lane == 0) {
      q_norm[row] = nq;
      k_norm[row] = nk;
    }
  }
}

// One row's input gradient: x the raw row, u the cotangent of the
// normalised row, norm the saved norm.
template <int NJ>
__device__ __forceinline__ void row_vjp(const float (&x)[4], const float (&u)[4], float norm, bool small_rows,
                                        void* out, size_t base, bool bf) {
  const float d = denom_of(norm);
  float z[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int j = 0; j < NJ; ++j) z[j] = __fmul_rn(-u[j], __fdiv_rn(__fdiv_rn(x[j], d), d));
  // the reference seeds each lane's accumulators with +0 + z (turns -0 into +0)
  const float g = row_sum(__fadd_rn(0.f, z[0]), __fadd_rn(0.f, z[1]), __fadd_rn(0.f, z[2]), __fadd_rn(0.f, z[3]),
                          small_rows);
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    const float direct = __fdiv_rn(u[j], d);
    const float unit = norm == 0.f ? 0.f : __fdiv_rn(x[j], norm);
    const float via_norm = norm >= 1e-12f ? __fmul_rn(g, unit) : 0.f;
    const float total = __fadd_rn(direct, via_norm);
    if (bf)
      static_cast<bf16*>(out)[base + 32 * j] = __float2bfloat16_rn(total);
    else
      static_cast<float*>(out)[base + 32 * j] = total;
  }
}

template <int K>
__global__ void __launch_bounds__(32 * kNormWarps) diag_norm_bwd_kernel(
    const void* __restrict__ q, const void* __restrict__ k, int in_bf16, const bf16* __restrict__ dq_memory,
    const float* __restrict__ dk_gain, const bf16* __restrict__ dk_memory, const float* __restrict__ q_norm,
    const float* __restrict__ k_norm, void* __restrict__ dq, void* __restrict__ dk, int64_t n_rows) {
  constexpr int NJ = K / 32;
  const bool bf = in_bf16 != 0, small_rows = n_rows < 16;
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * kNormWarps;
  for (int64_t row = (int64_t)blockIdx.x * kNormWarps + (threadIdx.x >> 5); row < n_rows; row += warps) {
    const size_t base = (size_t)row * K + lane;
    // every load of the row (q side and k side) requested before any arithmetic
    float xq[4] = {0.f, 0.f, 0.f, 0.f}, uq[4] = {0.f, 0.f, 0.f, 0.f};
    float xk[4] = {0.f, 0.f, 0.f, 0.f}, ug[4] = {0.f, 0.f, 0.f, 0.f}, um[4] = {0.f, 0.f, 0.f, 0.f};
    const bool has_k = dk_gain || dk_memory;
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      if (dq_memory) {
        xq[j] = load_f(q, base + 32 * j, bf);
        uq[j] = __bfloat162float(dq_memory[base + 32 * j]);
      }
      if (has_k) xk[j] = load_f(k, base + 32 * j, bf);
      if (dk_gain) ug[j] = dk_gain[base + 32 * j];
      if (dk_memory) um[j] = __bfloat162float(dk_memory[base + 32 * j]);
    }
    const float nq = dq_memory ? q_norm[row] : 0.f, nk = has_k ? k_norm[row] : 0.f;
    if (dq_memory) row_vjp<NJ>(xq, uq, nq, small_rows, dq, base, bf);
    if (has_k) {
      float u[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) u[j] = dk_gain && dk_memory ? __fadd_rn(ug[j], um[j]) : dk_gain ? ug[j] : um[j];
      row_vjp<NJ>(xk, u, nk, small_rows, dk, base, bf);
    }
  }
}

unsigned norm_grid(int64_t n_rows) {
  const int64_t blocks = (n_rows + kNormWarps - 1) / kNormWarps;
  const int64_t cap = 148 * 8 * 4;  // eight resident CTAs of 256 threads per SM, four waves of rows each
  return (unsigned)(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}

}  // namespace
}  // namespace kdn

using namespace kdn;

extern "C" {

int kdn_diag_norm_fwd(const void* q_raw, const void* k_raw, int in_bf16, void* q_memory, float* k_gain,
                      void* k_memory, float* q_norm, float* k_norm, int64_t n_rows, int64_t K,
                      kdn_stream_t stream) {
  if (n_rows < 0 || (K != 64 && K != 128))
    return set_error(KDN_ERR_INVALID, "kdn_diag_norm_fwd: n_rows >= 0 and K in {64, 128} required");
  if (n_rows == 0) return KDN_OK;
  if (!q_raw || !k_raw || !q_memory || !k_gain || !k_memory || !q_norm || !k_norm)
    return set_error(KDN_ERR_INVALID, "kdn_diag_norm_fwd: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  if (K == 128)
    diag_norm_fwd_kernel<128><<<norm_grid(n_rows), 32 * kNormWarps, 0, st>>>(
        q_raw, k_raw, in_bf16, static_cast<bf16*>(q_memory), k_gain, static_cast<bf16*>(k_memory), q_norm, k_norm,
        n_rows);
  else
    diag_norm_fwd_kernel<64><<<norm_grid(n_rows), 32 * kNormWarps, 0, st>>>(
        q_raw, k_raw, in_bf16, static_cast<bf16*>(q_memory), k_gain, static_cast<bf16*>(k_memory), q_norm, k_norm,
        n_rows);
  return check_launch("diag_norm_fwd_kernel");
}

int kdn_diag_norm_bwd(const void* q_raw, const void* k_raw, int in_bf16, const void* dq_memory,
                      const float* dk_gain, const void* dk_memory, const float* q_norm, const float* k_norm,
                      void* dq_raw, void* dk_raw, int64_t n_rows, int64_t K, kdn_stream_t stream) {
  if (n_rows < 0 || (K != 64 && K != 128))
    return set_error(KDN_ERR_INVALID, "kdn_diag_norm_bwd: n_rows >= 0 and K in {64, 128} required");
  if (n_rows == 0 || (!dq_memory && !dk_gain && !dk_memory)) return KDN_OK;
  if (!q_raw || !k_raw || !q_norm || !k_norm || (dq_memory && !dq_raw) || ((dk_gain || dk_memory) && !dk_raw))
    return set_error(KDN_ERR_INVALID, "kdn_diag_norm_bwd: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  const bf16* dqm = static_cast<const bf16*>(dq_memory);
  const bf16* dkm = static_cast<const bf16*>(dk_memory);
  if (K == 128)
    diag_norm_bwd_kernel<128><<<norm_grid(n_rows), 32 * kNormWarps, 0, st>>>(
        q_raw, k_raw, in_bf16, dqm, dk_gain, dkm, q_norm, k_norm, dq_raw, dk_raw, n_rows);
  else
    diag_norm_bwd_kernel<64><<<norm_grid(n_rows), 32 * kNormWarps, 0, st>>>(
        q_raw, k_raw, in_bf16, dqm, dk_gain, dkm, q_norm, k_norm, dq_raw, dk_raw, n_rows);
  return check_launch("diag_norm_bwd_kernel");
}

}  // extern "C"
