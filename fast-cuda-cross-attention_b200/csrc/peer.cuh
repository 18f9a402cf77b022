// Multi-GPU N_input split (config 4): the merge of the ranks' partial (m, l, O) triples as
// ONE kernel per rank over peer memory, instead of all-reduce(MAX) -> rescale ->
// all-reduce(SUM) -> divide through NCCL.
//
// Every rank owns one exchange buffer (a CUDA IPC allocation, mapped into every other
// rank's process over NVLink / NVSwitch; no multicast object is involved):
//
//   flags [64] u32 : [0, 8) "partials ready" epochs, [32, 40) "merge done" epochs, [63] a
//                    block counter of this rank's merge launch
//   pm [rows], pl [rows] : the rank's partial row maximum (natural-log units) and row sum
//   po [rows][dim]       : its unnormalised partial output, relative to pm
//   out [rows][dim]      : the merged, normalised output (every rank receives all rows)
//
// (each region starts on a 256-byte boundary).  Rank r's partial kernel writes pm / pl / po
// of its own buffer; then merge_kernel on every rank:
//   1. barrier "partials ready": each block's thread 0 stores the epoch into flags[rank] of
//      every rank's buffer (release, system scope) and waits until its own flags[0..n)
//      reach the epoch (acquire, system scope);
//   2. merges the rows [rank rows / n, (rank + 1) rows / n): M = max_p m_p,
//      L = sum_p e^(m_p - M) l_p, O = sum_p e^(m_p - M) O_p / L  (kernel_splitk.cu:186-236
//      upstream, across GPUs), reading every rank's po over NVLink, and stores each merged
//      row into the out region of every rank (the all-gather of the result, fused);
//   3. barrier "merge done", by the last block to finish (a counter in the flags): once it
//      passes, every rank has written its rows into this rank's out and finished reading
//      this rank's po, so the next call may overwrite both.
// Each wait is bounded (g_wait_ns); a wait that gives up records kTimeoutRank in the device
// status word and the kernel returns.  rank < 0 runs all ranks' rows in one launch without
// barriers (single-process emulation over buffers of one GPU, for tests).
#pragma once

#include "sm100.cuh"

namespace xattn {
namespace peer {

constexpr int kMaxRanks = 8;
constexpr int kThreads = 256;  // eight warps, one (row, column segment) each at a time
constexpr int kReadySlot = 0, kDoneSlot = 32, kCounterSlot = 63, kFlagWords = 64;

struct Layout {
  long long pm, pl, po, out, total;  // offsets and total size in 4-byte words
};

__host__ __device__ inline long long round_up64(long long n) { return (n + 63) / 64 * 64; }

__host__ __device__ inline Layout layout(long long rows, int dim) {
  Layout l;
  l.pm = kFlagWords;
  l.pl = l.pm + round_up64(rows);
  l.po = l.pl + round_up64(rows);
  l.out = l.po + round_up64(rows * dim);
  l.total = l.out + round_up64(rows * dim);
  return l;
}

struct Params {
  float* base[kMaxRanks];  // every rank's exchange buffer as mapped in this process
  long long rows;
  int dim, n_ranks, rank;  // rank < 0: emulation (all rows, no barriers)
  unsigned epoch;
  Layout lay;
};

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// base[i] for a run-time i without indexing the parameter array at run time (which would
// copy it to local memory)
__device__ __forceinline__ float* pick(float* const (&base)[kMaxRanks], int i) {
  float* r = base[0];
#pragma unroll
  for (int p = 1; p < kMaxRanks; ++p)
    if (i == p) r = base[p];
  return r;
}

// Barrier among the ranks on the flags at `slot`: announce the epoch to every rank, wait
// for every rank's announcement.  Called by one thread.
__device__ __forceinline__ bool rank_barrier(float* const (&base)[kMaxRanks], int n_ranks, int rank,
                                             unsigned epoch, int slot) {
  __threadfence_system();
#pragma unroll
  for (int p = 0; p < kMaxRanks; ++p)
    if (p < n_ranks) st_release_sys(reinterpret_cast<unsigned*>(base[p]) + slot + rank, epoch);
  const unsigned* f = reinterpret_cast<const unsigned*>(pick(base, rank)) + slot;
  const uint64_t t0 = global_ns();
  for (int p = 0; p < n_ranks; ++p) {
    while (static_cast<int>(ld_acquire_sys(f + p) - epoch) < 0) {
      if (global_ns() - t0 > g_wait_ns) {
        record_status(kTimeoutRank);
        return false;
      }
      __nanosleep(100);
    }
  }
  return true;
}

// One warp per unit = (row, segment of kSegCols columns), grid-stride over this rank's rows:
// lanes < n load the ranks' (m, l) while every lane issues its loads of the segment from ALL
// ranks (kSegVec float4 per lane per rank, the rank loop unrolled to kMaxRanks), so a unit
// costs one remote round trip whatever the rank count; the weights w_p = e^(m_p - M) / L come
// out of two shuffle reductions, and the merged segment is stored into every rank's out.
constexpr int kSegVec = 2;                  // float4 per lane per rank
constexpr int kSegCols = 32 * 4 * kSegVec;  // 256 columns per unit

__device__ __forceinline__ float4 fma4(float w, float4 x, float4 acc) {
  acc.x = fmaf(w, x.x, acc.x);
  acc.y = fmaf(w, x.y, acc.y);
  acc.z = fmaf(w, x.z, acc.z);
  acc.w = fmaf(w, x.w, acc.w);
  return acc;
}

__global__ void __launch_bounds__(kThreads) merge_kernel(const Params a) {
  __shared__ int go;
  const bool emulate = a.rank < 0;
  // launched as a programmatic dependent of the kernel that writes this rank's partials:
  // nothing below touches memory before that kernel has completed
  griddep_wait();
  if (threadIdx.x == 0) go = emulate ? 1 : rank_barrier(a.base, a.n_ranks, a.rank, a.epoch, kReadySlot);
  __syncthreads();
  const int n = a.n_ranks, lane = threadIdx.x % 32;
  const long long r0 = emulate ? 0 : a.rows * a.rank / n;
  const long long r1 = emulate ? a.rows : a.rows * (a.rank + 1) / n;
  const bool vec = (a.dim & 3) == 0;
  const int nseg = vec ? (a.dim + kSegCols - 1) / kSegCols : (a.dim + 31) / 32;
  const long long units = (r1 - r0) * nseg;
  const long long wpb = kThreads / 32;
  for (long long u = blockIdx.x * wpb + threadIdx.x / 32; go && u < units; u += gridDim.x * wpb) {
    const long long r = r0 + u / nseg;
    const int seg = static_cast<int>(u % nseg);
    const long long off = r * a.dim;
    float m = -INFINITY, l = 0.f;
    if (lane < n) {
      const float* bl = pick(a.base, lane);
      m = __ldcg(bl + a.lay.pm + r);
      l = __ldcg(bl + a.lay.pl + r);
    }
    if (vec) {
      float4 x[kMaxRanks][kSegVec];
#pragma unroll
      for (int p = 0; p < kMaxRanks; ++p)
#pragma unroll
        for (int j = 0; j < kSegVec; ++j) {
          const int c = seg * kSegCols + 4 * (lane + 32 * j);
          x[p][j] = p < n && c < a.dim ? __ldcg(reinterpret_cast<const float4*>(a.base[p] + a.lay.po + off + c))
                                       : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      if (!(m > -3.4028234663852886e38f)) m = -INFINITY;  // a rank without keys
      float mx = m;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float e = m > -INFINITY ? __expf(m - mx) : 0.f;
      float lsum = e * l;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
      const float w = lsum > 0.f ? e / lsum : 0.f;  // no keys anywhere: zeros
      float4 acc[kSegVec];
#pragma unroll
      for (int j = 0; j < kSegVec; ++j) acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int p = 0; p < kMaxRanks; ++p) {
        const float wp = __shfl_sync(0xffffffffu, w, p);  // 0 for p >= n
#pragma unroll
        for (int j = 0; j < kSegVec; ++j) acc[j] = fma4(wp, x[p][j], acc[j]);
      }
#pragma unroll
      for (int p = 0; p < kMaxRanks; ++p)
#pragma unroll
        for (int j = 0; j < kSegVec; ++j) {
          const int c = seg * kSegCols + 4 * (lane + 32 * j);
          if (p < n && c < a.dim) *reinterpret_cast<float4*>(a.base[p] + a.lay.out + off + c) = acc[j];
        }
    } else {
      const int c = seg * 32 + lane;
      float x[kMaxRanks];
#pragma unroll
      for (int p = 0; p < kMaxRanks; ++p) x[p] = p < n && c < a.dim ? __ldcg(a.base[p] + a.lay.po + off + c) : 0.f;
      if (!(m > -3.4028234663852886e38f)) m = -INFINITY;
      float mx = m;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float e = m > -INFINITY ? __expf(m - mx) : 0.f;
      float lsum = e * l;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
      const float w = lsum > 0.f ? e / lsum : 0.f;
      float acc = 0.f;
#pragma unroll
      for (int p = 0; p < kMaxRanks; ++p) acc = fmaf(__shfl_sync(0xffffffffu, w, p), x[p], acc);
#pragma unroll
      for (int p = 0; p < kMaxRanks; ++p)
        if (p < n && c < a.dim) a.base[p][a.lay.out + off + c] = acc;
    }
  }
  if (emulate) return;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();  // this block's rows are visible in every rank's buffer
    unsigned* counter = reinterpret_cast<unsigned*>(pick(a.base, a.rank)) + kCounterSlot;
    if (atomicAdd(counter, 1u) == gridDim.x - 1) {  // the last block of this launch
      *reinterpret_cast<volatile unsigned*>(counter) = 0u;  // for the next launch
      rank_barrier(a.base, a.n_ranks, a.rank, a.epoch, kDoneSlot);
    }
  }
}

}  // namespace peer
}  // namespace xattn
