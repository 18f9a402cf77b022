// Accurate fp32 mode (3xTF32): attention to fp32-level accuracy on the tcgen05 tensor cores.
//
//   S = Q K^T        3xTF32 batched GEMM (gemm3x_kernel, B operand K-major)
//   P = softmax(S / sqrt(D)) row by row, accurate expf, P normalised (softmax_rows_kernel)
//   O = P V          3xTF32 batched GEMM (B operand MN-major: V rows are keys)
//
// 3xTF32: every fp32 operand x is x_big + x_small with x_big = x truncated to TF32 (exactly
// what the tensor core reads when given x) and x_small = x - x_big (exact in fp32; the
// tensor core truncates it in turn, leaving an error of order 2^-22 |x|).  Each product is
// a.b ~ a.b_big + a.b_small + a_small.b_big, three kind::tf32 MMAs.  The two cross terms
// (about 2^-10 of the main product) accumulate in their own TMEM accumulator, so they are
// not aligned against the growing main sum at every step; the epilogue adds the two.  The residuals of Q, K, V are computed by split_residual_kernel and those of
// P by the softmax kernel; S and P live in the library workspace (B * N_latent * N_input
// floats each), so this mode trades HBM traffic for accuracy and is off by default.
//
// gemm3x_kernel: C[b] (M x N, row stride ldc) = A[b] (M x K, K-major) * B[b]^T (K-major:
// N x K) or A[b] * B[b] (MN-major: K x N).  One CTA per 128 x 128 output tile, K in chunks
// of 32 (one 128-byte swizzle row), a 3-stage TMA ring of (A, A_small, B, B_small) chunks
// (64 KB per stage), warp 0 TMA producer, warp 1 MMA issuer, warps 2..5 epilogue (TMEM ->
// registers -> global, bounds-checked).
#pragma once

#include "sm100.cuh"

namespace xattn {
namespace accurate {

constexpr int kTile = 128;
constexpr int kChunk = 32;                       // fp32 per 128-byte swizzle row
constexpr int kOpBytes = kTile * kChunk * 4;     // 16 KB: one operand chunk
constexpr int kStageBytes = 4 * kOpBytes;        // A, A_small, B, B_small
constexpr int kStages = 3;
constexpr int kSmemBytes = kStages * kStageBytes + 1024;
constexpr int kThreads = 192;
constexpr int kTmemCols = 256;  // main product at columns 0..127, cross terms at 128..255

struct GemmParams {
  CUtensorMap ta, tas, tb, tbs;  // A, A_small, B, B_small
  float* c;
  long long c_batch_stride;      // elements
  int ldc, m, n, k;
  int tiles_m, tiles_n;
};

// B operand K-major (B is N x K, rows contiguous along K) or MN-major (B is K x N, rows
// contiguous along N; loaded as four 32-column slabs in the "128-byte swizzle, 32-byte atom"
// layout, descriptor layout 1, SBO 512, LBO = slab stride).
template <bool kBMnMajor>
__global__ void __launch_bounds__(kThreads, 1) gemm3x_kernel(const __grid_constant__ GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  __shared__ __align__(8) uint64_t full[kStages], empty[kStages], acc_done;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int tiles = p.tiles_m * p.tiles_n;
  const int bz = blockIdx.x / tiles;
  const int tm = (blockIdx.x % tiles) / p.tiles_n;
  const int tn = blockIdx.x % p.tiles_n;
  const int m0 = tm * kTile, n0 = tn * kTile;
  const int n_chunks = (p.k + kChunk - 1) / kChunk;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    mbar_init(smem_u32(&acc_done), 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(&tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  volatile int* abort = &abort_flag;

  if (warp == 0) {
    if (elect_one()) {
      int s = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int c = 0; c < n_chunks && ok; ++c) {
        if (!(ok = mbar_wait(smem_u32(&empty[s]), phase ^ 1u, kTimeoutStageFree, abort))) break;
        const uint32_t st = smem_u32(smem + s * kStageBytes);
        const uint32_t fb = smem_u32(&full[s]);
        mbar_arrive_expect_tx(fb, kStageBytes);
        const int k0 = c * kChunk;
        tma_load_3d(st, &p.ta, fb, k0, m0, bz);
        tma_load_3d(st + kOpBytes, &p.tas, fb, k0, m0, bz);
        if (kBMnMajor) {  // {32 columns, 32 k rows, 4 slabs, batch}: slab index = n / 32
          tma_load_4d(st + 2 * kOpBytes, &p.tb, fb, 0, k0, n0 / kChunk, bz);
          tma_load_4d(st + 3 * kOpBytes, &p.tbs, fb, 0, k0, n0 / kChunk, bz);
        } else {
          tma_load_3d(st + 2 * kOpBytes, &p.tb, fb, k0, n0, bz);
          tma_load_3d(st + 3 * kOpBytes, &p.tbs, fb, k0, n0, bz);
        }
        if (++s == kStages) { s = 0; phase ^= 1u; }
      }
      for (int i = 0; i < kStages; ++i) {  // no copy in flight at exit
        if (--s < 0) { s = kStages - 1; phase ^= 1u; }
        mbar_wait(smem_u32(&empty[s]), phase, kTimeoutDrain, abort);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      int s = 0;
      uint32_t phase = 0;
      const uint32_t idesc = instr_desc(2, kTile, kTile, false, kBMnMajor);
      for (int c = 0; c < n_chunks; ++c) {
        if (!mbar_wait(smem_u32(&full[s]), phase, kTimeoutTmaFull, abort)) break;
        tc_fence_after();
        const uint32_t st = smem_u32(smem + s * kStageBytes);
#pragma unroll
        for (int kk = 0; kk < kChunk / 8; ++kk) {
          const uint64_t a = smem_desc(st + kk * 32, 16, 1024, kSw128);
          const uint64_t as = smem_desc(st + kOpBytes + kk * 32, 16, 1024, kSw128);
          uint64_t b, bs;
          if (kBMnMajor) {
            b = smem_desc(st + 2 * kOpBytes + kk * 1024, 4096, 512, kSw128Atom32);
            bs = smem_desc(st + 3 * kOpBytes + kk * 1024, 4096, 512, kSw128Atom32);
          } else {
            b = smem_desc(st + 2 * kOpBytes + kk * 32, 16, 1024, kSw128);
            bs = smem_desc(st + 3 * kOpBytes + kk * 32, 16, 1024, kSw128);
          }
          mma_tf32_ss(tmem + kTile, as, b, idesc, (c | kk) != 0);
          mma_tf32_ss(tmem + kTile, a, bs, idesc, 1);
          mma_tf32_ss(tmem, a, b, idesc, (c | kk) != 0);
        }
        mma_commit(smem_u32(&empty[s]));
        if (++s == kStages) { s = 0; phase ^= 1u; }
      }
      mma_commit(smem_u32(&acc_done));
    }
  } else {
    const int quad = warp & 3;
    const int row = m0 + quad * 32 + lane;
    const uint32_t t_row = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    if (warp_mbar_wait(smem_u32(&acc_done), 0, kTimeoutMmaDone, abort)) {
      tc_fence_after();
      float* dst = p.c + bz * p.c_batch_stride + static_cast<long long>(row) * p.ldc + n0;
      for (int cc = 0; cc < kTile / 32; ++cc) {
        uint32_t v[32], w[32];
        tmem_ld32(t_row + cc * 32, v);
        tmem_ld32(t_row + kTile + cc * 32, w);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) + __uint_as_float(w[i]));
        if (row < p.m) {
          const int base = n0 + cc * 32;
          if (base + 32 <= p.n && (p.ldc & 3) == 0) {
            float4* d4 = reinterpret_cast<float4*>(dst + cc * 32);
#pragma unroll
            for (int i = 0; i < 8; ++i)
              d4[i] = make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                                  __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3]));
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (base + i < p.n) dst[cc * 32 + i] = __uint_as_float(v[i]);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (abort_flag) {  // stable here: every give_up preceded the barrier
    settle_after_give_up();
    __syncthreads();
  }
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, kTmemCols);
}

// x_small = x - trunc_tf32(x), elementwise (exact in fp32).
__global__ void __launch_bounds__(256) split_residual_kernel(const float* __restrict__ x,
                                                             float* __restrict__ small, long long n) {
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float v = x[i];
    small[i] = v - __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
  }
}

// Row softmax of S (rows of `cols` scores, row stride ld) in place into P, with P's TF32
// residual into ps: P = exp(scale (s - max)) / sum, accurate expf, one warp per row.
__global__ void __launch_bounds__(256) softmax_rows_kernel(float* __restrict__ s,
                                                           float* __restrict__ ps, long long rows,
                                                           int cols, int ld, float scale) {
  const long long r = static_cast<long long>(blockIdx.x) * 8 + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (r >= rows) return;
  float* row = s + r * ld;
  float* rs = ps + r * ld;
  float mx = -INFINITY;
  for (int c = lane; c < cols; c += 32) mx = fmaxf(mx, row[c]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.f;
  for (int c = lane; c < cols; c += 32) {
    const float e = expf(scale * (row[c] - mx));
    row[c] = e;
    sum += e;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float inv = 1.f / sum;
  for (int c = lane; c < cols; c += 32) {
    const float pv = row[c] * inv;
    row[c] = pv;
    rs[c] = pv - __uint_as_float(__float_as_uint(pv) & 0xFFFFE000u);
  }
}

}  // namespace accurate
}  // namespace xattn
