// Generic CUDA-core kernels: the shape-agnostic attention path (any D, any key range,
// fp32 / fp16 / bf16 inputs, strided per-head views), the log-sum-exp combine of split
// partials (upstream kernel_splitk.cu:186-236) and the helpers of the multi-GPU merge.
//
// The generic attention kernel is the GPU path for shapes the tcgen05 kernels do not
// take (D not a multiple of 64, D > 768, ...).  It is correct for every shape and never
// used where a tensor-core kernel applies.  One warp owns one query row; keys are
// consumed one at a time with an online softmax in the log2 domain; the query row and
// the output accumulator live in shared memory so D is bounded only by shared memory.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "sm100.cuh"

namespace xattn {
namespace simt {

__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ void from_f(float* d, float x) { *d = x; }
__device__ __forceinline__ void from_f(__nv_bfloat16* d, float x) { *d = __float2bfloat16_rn(x); }

template <typename Tin, typename Tout>
struct Args {
  const Tin* q;
  const Tin* k;
  const Tin* v;
  Tout* out;          // final mode
  float* po;          // split mode: [B*H][Nl][S][dh] (flattened like the upstream layout)
  float* pm;
  float* pl;
  long long q_bs, k_bs, o_bs;  // batch strides (elements)
  int ld_q, ld_k, ld_o;        // row strides (elements)
  int heads, dh;               // head h reads columns [h*dh, (h+1)*dh)
  int n_latent, n_input;
  int num_splits, split_chunk, split_mode;
  float scale_log2;            // log2(e) * softmax scale
};

constexpr int kWarps = 4;

template <typename Tin, typename Tout>
__global__ void __launch_bounds__(kWarps * 32) attention_kernel(const Args<Tin, Tout> a) {
  extern __shared__ float sm[];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int row = blockIdx.x * kWarps + warp;
  const int bh = blockIdx.y;
  const int split = blockIdx.z;
  const int b = bh / a.heads, hd = bh % a.heads;
  float* qs = sm + warp * 2 * a.dh;
  float* os = qs + a.dh;
  const bool live = row < a.n_latent;
  const int k0 = split * a.split_chunk;
  const int k1 = min(k0 + a.split_chunk, a.n_input);
  if (live) {
    const Tin* qr = a.q + b * a.q_bs + static_cast<long long>(row) * a.ld_q + hd * a.dh;
    for (int d = lane; d < a.dh; d += 32) {
      qs[d] = to_f(qr[d]);
      os[d] = 0.f;
    }
  }
  __syncwarp();
  float m = -INFINITY, l = 0.f;
  if (live) {
    for (int key = k0; key < k1; ++key) {
      const Tin* kr = a.k + b * a.k_bs + static_cast<long long>(key) * a.ld_k + hd * a.dh;
      float dot = 0.f;
      for (int d = lane; d < a.dh; d += 32) dot = fmaf(qs[d], to_f(kr[d]), dot);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
      const float t = dot * a.scale_log2;
      const float mn = fmaxf(m, t);
      const float alpha = exp2f(m - mn);
      const float pw = exp2f(t - mn);
      l = l * alpha + pw;
      m = mn;
      const Tin* vr = a.v + b * a.k_bs + static_cast<long long>(key) * a.ld_k + hd * a.dh;
      for (int d = lane; d < a.dh; d += 32) os[d] = fmaf(os[d], alpha, pw * to_f(vr[d]));
    }
  }
  __syncwarp();
  if (!live) return;
  if (a.split_mode) {
    const size_t pidx = (static_cast<size_t>(bh) * a.n_latent + row) * a.num_splits + split;
    float* dst = a.po + pidx * a.dh;
    if (k1 > k0) {
      for (int d = lane; d < a.dh; d += 32) dst[d] = os[d];
      if (lane == 0) {
        a.pm[pidx] = m * 0.69314718055994531f;
        a.pl[pidx] = l;
      }
    } else {
      for (int d = lane; d < a.dh; d += 32) dst[d] = 0.f;
      if (lane == 0) {
        a.pm[pidx] = -3.4028234663852886e38f;
        a.pl[pidx] = 0.f;
      }
    }
  } else {
    const float inv = 1.f / l;
    Tout* dst = a.out + b * a.o_bs + static_cast<long long>(row) * a.ld_o + hd * a.dh;
    for (int d = lane; d < a.dh; d += 32) from_f(&dst[d], os[d] * inv);
  }
}

// Log-sum-exp merge of S split partials per row (upstream kernel_splitk.cu:186-236):
// M = max_s m_s; L = sum_s e^(m_s-M) l_s; O = sum_s e^(m_s-M) O_s / L.  Splits whose m is
// -FLT_MAX (empty) get weight 0.  One thread per (row, four columns): the partial outputs do
// not depend on the weights, so the thread issues its loads of up to kCombineChunk splits'
// outputs together with their (m, l) and only then forms the weights -- one memory round trip
// per chunk of splits, merged across chunks with a running maximum (online log-sum-exp).  No
// shared memory, no block barrier.  kPartial: write the merged partial instead of the
// normalised output -- O_u = sum_s e^(m_s-M) O_s (unnormalised) to out, M to pm_out and L to
// pl_out (a row with no keys keeps the empty-split triple -FLT_MAX, 0, 0).
// po rows: [rows][S][dim] (the upstream layout).
constexpr int kCombineThreads = 256;
constexpr int kCombineChunk = 4;

template <typename Tout, bool kPartial = false>
__global__ void __launch_bounds__(kCombineThreads) combine_kernel(const float* __restrict__ po,
                                                                  const float* __restrict__ pm,
                                                                  const float* __restrict__ pl,
                                                                  Tout* __restrict__ out,
                                                                  long long rows, int dim,
                                                                  int num_splits, int ld_o,
                                                                  float* __restrict__ pm_out = nullptr,
                                                                  float* __restrict__ pl_out = nullptr) {
  // a dependent launched with programmatic serialization (the multi-GPU merge) may take free
  // SM slots now; it waits in griddep_wait() for this grid's results
  griddep_launch_dependents();
  griddep_wait();  // launched as a programmatic dependent of the kernel writing the partials
  constexpr float kEmpty = -3.4028234663852886e38f;
  const int S = num_splits;
  // float4 loads need 16-byte aligned rows: dim % 4 == 0 and an aligned po (caller scratch of
  // the upstream split entry may be any float pointer); otherwise one column per thread
  const bool vec = (dim & 3) == 0 && (reinterpret_cast<uintptr_t>(po) & 15) == 0;
  const int w = vec ? 4 : 1;              // columns per thread
  const int per_row = (dim + w - 1) / w;  // threads per row
  const long long idx = static_cast<long long>(blockIdx.x) * kCombineThreads + threadIdx.x;
  if (idx >= rows * per_row) return;
  const long long r = idx / per_row;
  const int c = static_cast<int>(idx - r * per_row) * w;
  const float* src = po + r * S * static_cast<long long>(dim) + c;
  const float* m = pm + r * S;
  const float* l = pl + r * S;
  float mx = -INFINITY, lsum = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s0 = 0; s0 < S; s0 += kCombineChunk) {
    float4 x[kCombineChunk];
    float ms[kCombineChunk], ls[kCombineChunk];
#pragma unroll
    for (int j = 0; j < kCombineChunk; ++j) {
      const bool in = s0 + j < S;
      const float* row = src + static_cast<long long>(s0 + j) * dim;
      if (vec)
        x[j] = in ? *reinterpret_cast<const float4*>(row) : make_float4(0.f, 0.f, 0.f, 0.f);
      else
        x[j] = make_float4(in ? row[0] : 0.f, 0.f, 0.f, 0.f);
      ms[j] = in ? m[s0 + j] : kEmpty;
      ls[j] = in ? l[s0 + j] : 0.f;
    }
    float cm = mx;
#pragma unroll
    for (int j = 0; j < kCombineChunk; ++j)
      if (ms[j] > kEmpty) cm = fmaxf(cm, ms[j]);
    if (cm == -INFINITY) continue;  // nothing but empty splits so far
    const float f = __expf(mx - cm);  // 0 while mx is still -inf
    lsum *= f;
    acc.x *= f;
    acc.y *= f;
    acc.z *= f;
    acc.w *= f;
#pragma unroll
    for (int j = 0; j < kCombineChunk; ++j) {
      const float e = ms[j] > kEmpty ? __expf(ms[j] - cm) : 0.f;
      lsum = fmaf(e, ls[j], lsum);
      acc.x = fmaf(e, x[j].x, acc.x);
      acc.y = fmaf(e, x[j].y, acc.y);
      acc.z = fmaf(e, x[j].z, acc.z);
      acc.w = fmaf(e, x[j].w, acc.w);
    }
    mx = cm;
  }
  const float inv = kPartial ? 1.f : (lsum > 0.f ? 1.f / lsum : 0.f);  // no keys: zeros
  if (kPartial && c == 0) {
    pm_out[r] = lsum > 0.f ? mx : kEmpty;
    pl_out[r] = lsum;
  }
  Tout* dst = out + r * static_cast<long long>(ld_o) + c;
  const float v[4] = {acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv};
  for (int e = 0; e < w; ++e)
    if (c + e < dim) from_f(&dst[e], v[e]);
}

// Multi-GPU N_input split, step 2: after an all-reduce MAX of the row maxima into
// `mglob`, rescale this rank's partial to the global max in place:
//   O <- O * e^(m - M),  l <- l * e^(m - M).
// Rows are packed as [rows][dim + 1] with l in the last column, so one SUM all-reduce
// merges O and l together.
__global__ void __launch_bounds__(128) lse_rescale_kernel(float* __restrict__ ol,
                                                          const float* __restrict__ m_local,
                                                          const float* __restrict__ m_glob,
                                                          long long rows, int dim) {
  const long long r = static_cast<long long>(blockIdx.x) * 4 + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (r >= rows) return;
  const float ml = m_local[r];
  const float f = ml > -3.4028234663852886e38f ? __expf(ml - m_glob[r]) : 0.f;
  float* row = ol + r * (dim + 1);
  for (int d = lane; d <= dim; d += 32) row[d] *= f;
}

// Multi-GPU N_input split, step 4: out = O / l from the summed [rows][dim + 1] buffer.
__global__ void __launch_bounds__(128) lse_finalize_kernel(const float* __restrict__ ol,
                                                           float* __restrict__ out,
                                                           long long rows, int dim) {
  const long long r = static_cast<long long>(blockIdx.x) * 4 + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (r >= rows) return;
  const float* row = ol + r * (dim + 1);
  const float inv = 1.f / row[dim];
  for (int d = lane; d < dim; d += 32) out[r * dim + d] = row[d] * inv;
}

// Pack split-mode partials (po [rows][dim], pl [rows]) into [rows][dim + 1].
__global__ void __launch_bounds__(128) lse_pack_kernel(const float* __restrict__ po,
                                                       const float* __restrict__ pl,
                                                       float* __restrict__ ol, long long rows,
                                                       int dim) {
  const long long r = static_cast<long long>(blockIdx.x) * 4 + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (r >= rows) return;
  for (int d = lane; d < dim; d += 32) ol[r * (dim + 1) + d] = po[r * dim + d];
  if (lane == 0) ol[r * (dim + 1) + dim] = pl[r];
}

// Empty partials (no keys in the range, upstream kernel_splitk.cu:62-71): pm = -FLT_MAX,
// pl = 0, po = 0 for `n` (row, split) entries of `dim` columns.
__global__ void __launch_bounds__(256) empty_partials_kernel(float* __restrict__ po, float* __restrict__ pm,
                                                             float* __restrict__ pl, long long n, int dim) {
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    pm[i] = -3.4028234663852886e38f;
    pl[i] = 0.f;
  }
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n * dim; i += stride)
    po[i] = 0.f;
}

// Widen fp16 to fp32 (exact: every fp16 value is representable in fp32, and in TF32), 8
// elements per thread per step.  n8 = number of 8-element groups; in and out 16-byte aligned.
__global__ void __launch_bounds__(256) widen_half_kernel(const uint4* __restrict__ in,
                                                         float4* __restrict__ out, long long n8) {
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const uint4 v = in[i];
    const __half2* h = reinterpret_cast<const __half2*>(&v);
    const float2 a = __half22float2(h[0]), b = __half22float2(h[1]);
    const float2 c = __half22float2(h[2]), d = __half22float2(h[3]);
    out[2 * i] = make_float4(a.x, a.y, b.x, b.y);
    out[2 * i + 1] = make_float4(c.x, c.y, d.x, d.y);
  }
}

}  // namespace simt
}  // namespace xattn
