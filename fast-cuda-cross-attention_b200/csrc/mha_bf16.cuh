// Multi-head bf16 cross attention on tcgen05 (kind::f16: bf16 operands, fp32 accumulation).
//
// O[b, i, h*dh : (h+1)*dh] = softmax_j(Q_h[b, i] . K_h[b, j] / sqrt(dh)) V_h[b, j], with the
// heads side by side in each row (row stride heads * dh), bf16 in and out.  This is the
// per-head restatement of the upstream computation (generate_references.py:17-23 applied to
// each head's columns); there is no upstream bf16 kernel.
//
// One CTA owns 128 query rows of one (batch, head); a head dimension of at most 128 leaves
// TMEM room for two CTAs per SM (256 columns each: two S tiles of 64 keys at columns 0..127,
// O at 128..128+dh), so the two CTAs' softmax and tensor phases overlap without any cross-CTA
// protocol.  S is double-buffered in TMEM (columns 0..63 and 64..127).  The softmax warps
// write P (bf16, two per 32-bit column) over the first 32 columns of its own S buffer, and
// P V reads A from TMEM (tcgen05.mma .ts form); tcgen05 MMAs issued by one thread execute in
// issue order, so Q K^T of tile t+2, issued after P V of tile t, overwrites that buffer
// only after P V consumed it.  Per CTA:
//   warp 0      TMA producer: Q once per item (resident), then K and V tiles of 64 keys
//               through a ring in the order K(0), then per tile K(j+1), V(j)
//   warp 1      MMA issuer: S = Q K^T (M=128, N=64, K=dh), O += P V (M=128, N=dh, K=64)
//   warps 2..5  softmax, one query row per thread (warp w reads TMEM lanes 32*(w%4)..+31),
//               then the epilogue: O / l in bf16 through per-warp staging slots in shared
//               memory, written out by TMA stores (32 x 32 boxes) that run while the warps
//               start the next item; stores of one row per thread took ~1.8 us per item
// Persistent: two CTAs per SM loop over the (batch, head, 128-row block) items, keeping TMEM,
// barriers and the ring across items; the next item's Q load and first Q K^T overlap the
// current item's epilogue.
// Operands in shared memory, in boxes of bc columns: bc = 64 (128-byte swizzle rows) when d
// is a multiple of 64, else bc = 32 (64-byte swizzle rows), so every box lies inside the
// head.  (At d = 96, two 64-column boxes with the next head's columns unused measured 1 %
// faster at equal ring depth, but leave no room for the output staging.)
//   Q   K-major, dh/bc boxes of 128 rows x bc columns
//   K   K-major, boxes of 64 keys x bc columns
//   V   MN-major (rows are keys): the same boxes; the descriptor walks keys in 8-row groups
//       (SBO = 8 rows) and head columns in bc-wide groups (LBO = one box)
// Q, the ring and the output staging share a 112 KB operand area; the ring takes as many
// stages as fit (four at d = 128, five at d = 96, kMaxStages at d = 32 and 64).  The barriers live after it: with no static
// shared memory the dynamic region starts 1024-byte aligned (checked at run time), which
// leaves room for two CTAs per SM.
// Row sums on the tensor core (kTcSum, d <= 112): with each P.V step the MMA issuer also
// multiplies P by an all-ones B operand (N = 16), accumulating l = sum_k P[r, k] of the
// bf16-rounded weights into TMEM columns 128+d .. 143+d; the softmax warps then do no
// per-score summation.  The ones operand is a single 128-byte no-swizzle core matrix read
// with zero strides, valid because every element of the operand is the same.
#pragma once

#include <cuda_bf16.h>

#include "sm100.cuh"

namespace xattn {
namespace mha {

constexpr int kRows = 128;
constexpr int kKeys = 64;
// Operand area: Q (resident per item) followed by the K/V ring, whose stage count follows
// from the head dimension's tile size (kMaxStages at most).
constexpr int kOperandBytes = 112 * 1024;
constexpr int kMaxStages = 8;
constexpr int kBarOffset = kOperandBytes;
constexpr int kOnesOffset = kBarOffset + 256;   // 8 rows x 16 B of bf16 ones
constexpr int kSmemBytes = kOnesOffset + 128;
constexpr int kThreads = 192;
constexpr int kSoftmaxWarps = 4;
constexpr int kTmemCols = 256;
constexpr int kSCol = 0;
constexpr int kOCol = 128;
constexpr float kRescaleLog2 = 8.f;  // lazy rescale threshold (log2 units), as the fp32 kernels

struct Params {
  CUtensorMap tq, tk, tv;  // boxes of Layout<dh>::kBc columns x (128 or kKeys) rows
  CUtensorMap to;          // output, boxes of 32 columns x 32 rows, 64-byte swizzle
  int heads, n_latent, n_input, dh, ld;  // ld = heads * dh elements per row
  int n_row_blocks;
  int n_items;                           // B * heads * n_row_blocks
  float scale_log2;
};

__host__ __device__ constexpr bool supports_dh(int dh) {
  return dh == 32 || dh == 64 || dh == 96 || dh == 128;
}

struct __align__(8) Barriers {
  uint64_t q_full;      // Q of the current item landed
  uint64_t q_empty;     // the current item's last Q K^T completed (Q buffer free)
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t s_full[2];  // S buffer b holds the scores of tile j (j % 2 == b)
  uint64_t p_full[2];   // P of tile g is in TMEM (over its S): barrier g % 2.  One per S
                        // buffer: Q K^T of tile g + 1 is issued before P V of tile g, so a
                        // warp can finish tile g + 1 while another is still on tile g; with a
                        // single counter its second arrival would complete tile g's phase
  uint64_t pv_done;     // O += P V of the current tile completed (O current)
  uint64_t o_done;      // last P V completed
  uint32_t tmem_slot;
  int abort_flag;
};
static_assert(sizeof(Barriers) <= 256, "barrier block exceeds its reserved bytes");

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

__host__ __device__ constexpr bool tc_sum_for(int dh) { return dh <= 112; }

// Compile-time operand layout of one head dimension (the MMA issuer is a single thread on
// the tensor pipe's critical path: its per-step address arithmetic must fold to constants).
template <int kDh>
struct Layout {
  static constexpr bool kTcSum = tc_sum_for(kDh);
  static constexpr int kBc = kDh % 64 == 0 ? 64 : 32;        // columns per box
  static constexpr int kRowB = 2 * kBc;                      // bytes per swizzle row
  static constexpr uint32_t kSwz = kRowB == 128 ? kSw128 : kSw64;
  static constexpr int kBoxes = (kDh + kBc - 1) / kBc;
  static constexpr int kQBox = kRows * kRowB;
  static constexpr int kKvBox = kKeys * kRowB;
  static constexpr int kStageBytes = kBoxes * kKvBox;
  static constexpr int kQBytes = kBoxes * kQBox;
  // Output staging: per softmax warp, slots of 32 rows x 32 columns (2 KB) for the TMA
  // store; a slot per 32-column chunk when the ring still keeps 5 stages, else two.
  static constexpr int kChunks = kDh / 32;
  static constexpr int kChunkBytes = 32 * 64;
  static constexpr int kSlots =
      (kOperandBytes - kQBytes - kSoftmaxWarps * kChunks * kChunkBytes) / kStageBytes >= 5 ? kChunks : 2;
  static constexpr int kStagingBytes = kSoftmaxWarps * kSlots * kChunkBytes;
  static constexpr int kStages = (kOperandBytes - kQBytes - kStagingBytes) / kStageBytes < kMaxStages
                                     ? (kOperandBytes - kQBytes - kStagingBytes) / kStageBytes
                                     : kMaxStages;
  static constexpr int kStagingOffset = kQBytes + kStages * kStageBytes;
  static_assert(kStagingOffset + kStagingBytes <= kOperandBytes, "operand area overflow");
  static constexpr int kKStepsBox = kBc / 16;                // K steps of 16 per swizzle row
  static_assert(kStages >= 2, "K/V ring needs two stages");
};

template <int kDh>
__global__ void __launch_bounds__(kThreads, 2) mha_bf16_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  // swizzled TMA boxes and UMMA descriptors need 1024-byte alignment; the kernel has no
  // static shared memory, so the dynamic region starts at the window base.  Checked anyway:
  // a misaligned region records a status code and the CTA does nothing (uniform exit).
  if ((smem_u32(smem) & 1023u) != 0) {
    if (threadIdx.x == 0) record_status(kMisalignedSmem);
    return;
  }
  uint8_t* qs = smem;
  using L = Layout<kDh>;
  constexpr bool kTcSum = L::kTcSum;
  constexpr int rowb = L::kRowB, n_boxes = L::kBoxes, q_box = L::kQBox, kv_box = L::kKvBox;
  constexpr int stage_bytes = L::kStageBytes, n_stages = L::kStages;
  constexpr uint32_t swz = L::kSwz;
  uint8_t* stages = smem + L::kQBytes;
  const uint32_t staging = smem_u32(smem + L::kStagingOffset);
  Barriers& bars = *reinterpret_cast<Barriers*>(smem + kBarOffset);
  uint32_t& tmem_slot = bars.tmem_slot;
  int& abort_flag = bars.abort_flag;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int n_tiles = (p.n_input + kKeys - 1) / kKeys;  // >= 1: the host skips N_input == 0
  // Persistent: this CTA takes items blockIdx.x, blockIdx.x + gridDim.x, ...  The tile loop
  // runs on a global tile index g = (local item count) * n_tiles + j, which picks the S
  // buffer and the parity of every per-tile barrier; per-item barriers use the item count.
  struct Item {
    int row0, col0, b;
  };
  auto item_at = [&](int item) {
    const int rb = item % p.n_row_blocks, bh = item / p.n_row_blocks;
    return Item{rb * kRows, (bh % p.heads) * kDh, bh / p.heads};
  };
  if (threadIdx.x == 0) XATTN_TRACE_POINT(14, 0);

  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(smem_u32(&bars.q_full), 1);
    mbar_init(smem_u32(&bars.q_empty), 1);
    for (int s = 0; s < n_stages; ++s) {
      mbar_init(smem_u32(&bars.full[s]), 1);
      mbar_init(smem_u32(&bars.empty[s]), 1);
    }
    for (int i = 0; i < 2; ++i) mbar_init(smem_u32(&bars.s_full[i]), 1);
    for (int i = 0; i < 2; ++i) mbar_init(smem_u32(&bars.p_full[i]), kSoftmaxWarps);
    mbar_init(smem_u32(&bars.pv_done), 1);
    mbar_init(smem_u32(&bars.o_done), 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(&tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  if (kTcSum && warp == 2) {  // the ones operand: 64 bf16 of 1.0, for the tensor core
    reinterpret_cast<uint32_t*>(smem + kOnesOffset)[lane] = 0x3F803F80u;
    fence_proxy_async_smem();
  }
  if (warp == 1 && lane == 0) {
    tma_prefetch_desc(&p.tq);
    tma_prefetch_desc(&p.tk);
    tma_prefetch_desc(&p.tv);
    tma_prefetch_desc(&p.to);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  volatile int* abort = &abort_flag;

  if (warp == 0) {
    // ============================================================== TMA producer
    if (elect_one()) {
      int s = 0;
      uint32_t phase = 0;
      bool ok = true;
      int it = 0;
      for (int item = blockIdx.x; item < p.n_items && ok; item += gridDim.x, ++it) {
        const Item w = item_at(item);
        // the Q buffer is free once the previous item's last Q K^T completed
        if (it > 0 && !(ok = mbar_wait(smem_u32(&bars.q_empty), (it - 1) & 1, kTimeoutStageFree, abort)))
          break;
        mbar_arrive_expect_tx(smem_u32(&bars.q_full), n_boxes * q_box);
        for (int c = 0; c < n_boxes; ++c)
          tma_load_3d(smem_u32(qs + c * q_box), &p.tq, smem_u32(&bars.q_full),
                      w.col0 + c * L::kBc, w.row0, w.b);
        auto load = [&](const CUtensorMap* map, int tile) {
          if (!(ok = mbar_wait(smem_u32(&bars.empty[s]), phase ^ 1u, kTimeoutStageFree, abort))) return;
          mbar_arrive_expect_tx(smem_u32(&bars.full[s]), stage_bytes);
          for (int c = 0; c < n_boxes; ++c)
            tma_load_3d(smem_u32(stages + s * stage_bytes + c * kv_box), map,
                        smem_u32(&bars.full[s]), w.col0 + c * L::kBc, tile * kKeys, w.b);
          if (++s == n_stages) { s = 0; phase ^= 1u; }
        };
        load(&p.tk, 0);
        for (int j = 0; j < n_tiles && ok; ++j) {
          if (j + 1 < n_tiles) load(&p.tk, j + 1);
          if (ok) load(&p.tv, j);
        }
      }
      // every stage loaded is released by an MMA commit; wait for the last ones (and the
      // last Q) so no copy is in flight at exit
      for (int i = 0; i < n_stages; ++i) {
        if (--s < 0) { s = n_stages - 1; phase ^= 1u; }
        mbar_wait(smem_u32(&bars.empty[s]), phase, kTimeoutDrain, abort);
      }
      if (it > 0) mbar_wait(smem_u32(&bars.q_full), (it - 1) & 1, kTimeoutDrain, abort);
    }
  } else if (warp == 1) {
    // ============================================================== MMA issuer
    if (elect_one()) {
      int s = 0;
      uint32_t phase = 0;
      bool ok = true;
      const uint32_t idesc_qk = instr_desc(1, kRows, kKeys, false, false);
      constexpr uint32_t idesc_pv = instr_desc(1, kRows, kDh, false, true);
      const uint32_t idesc_sum = instr_desc(1, kRows, 16, false, false);
      const uint64_t ones_desc = smem_desc(smem_u32(smem + kOnesOffset), 0, 0, kSwNone);
      constexpr int ksteps_qk = kDh / 16;
      constexpr int ksteps_box = L::kKStepsBox;
      int it = 0;
      for (int item = blockIdx.x; item < p.n_items && ok; item += gridDim.x, ++it) {
        const int g0 = it * n_tiles;
        if (!(ok = mbar_wait(smem_u32(&bars.q_full), it & 1, kTimeoutTmaFull, abort))) break;
        tc_fence_after();
        auto mma_qk = [&](int j) {  // S of tile g0 + j into buffer (g0 + j) % 2
          if (!(ok = mbar_wait(smem_u32(&bars.full[s]), phase, kTimeoutTmaFull, abort))) return;
          tc_fence_after();
          const uint32_t st = smem_u32(stages + s * stage_bytes);
#pragma unroll
          for (int ks = 0; ks < ksteps_qk; ++ks) {
            const int c = ks / ksteps_box, off = (ks % ksteps_box) * 32;
            const uint64_t ad = smem_desc(smem_u32(qs) + c * q_box + off, 16, 8 * rowb, swz);
            const uint64_t bd = smem_desc(st + c * kv_box + off, 16, 8 * rowb, swz);
            mma_f16_ss(tmem + kSCol + ((g0 + j) & 1) * kKeys, ad, bd, idesc_qk, ks != 0);
          }
          mma_commit(smem_u32(&bars.empty[s]));
          mma_commit(smem_u32(&bars.s_full[(g0 + j) & 1]));
          if (j == n_tiles - 1) mma_commit(smem_u32(&bars.q_empty));  // Q no longer read
          if (++s == n_stages) { s = 0; phase ^= 1u; }
        };
        // buffer (g0 + j) % 2 last held P of tile g0 + j - 2, read by a P V issued earlier
        mma_qk(0);
        for (int j = 0; j < n_tiles && ok; ++j) {
          const int g = g0 + j;
          if (j + 1 < n_tiles) {
            mma_qk(j + 1);
            if (!ok) break;
          }
          // P of tile g; for j == 0 also: the epilogue of the previous item read O
          if (!(ok = mbar_wait(smem_u32(&bars.p_full[g & 1]), (g >> 1) & 1, kTimeoutSoftmax, abort)))
            break;
          if (!(ok = mbar_wait(smem_u32(&bars.full[s]), phase, kTimeoutTmaFull, abort))) break;
          tc_fence_after();
          const uint32_t st = smem_u32(stages + s * stage_bytes);
#pragma unroll
          for (int ks = 0; ks < kKeys / 16; ++ks) {
            const uint32_t a_tmem = tmem + kSCol + (g & 1) * kKeys + ks * 8;  // 16 keys of P
            // V MN-major: 16 keys = 16 swizzle rows; head columns step by a box (LBO)
            const uint64_t bd = smem_desc(st + ks * 16 * rowb, kv_box, 8 * rowb, swz);
            mma_f16_ts(tmem + kOCol, a_tmem, bd, idesc_pv, (j | ks) != 0);
            if (kTcSum) mma_f16_ts(tmem + kOCol + kDh, a_tmem, ones_desc, idesc_sum, (j | ks) != 0);
          }
          mma_commit(smem_u32(&bars.empty[s]));
          mma_commit(smem_u32(&bars.pv_done));
          if (++s == n_stages) { s = 0; phase ^= 1u; }
        }
        mma_commit(smem_u32(&bars.o_done));
      }
    }
  } else {
    // ============================================================== softmax + epilogue
    const int quad = warp & 3;
    const uint32_t t_row = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    bool ok = true;
    int it = 0;
    for (int item = blockIdx.x; item < p.n_items && ok; item += gridDim.x, ++it) {
      const Item wi = item_at(item);
      const int g0 = it * n_tiles;
      float m_run = -INFINITY;
      float l_run = 0.f;
      for (int j = 0; j < n_tiles; ++j) {
        const int g = g0 + j;
        const int valid = min(kKeys, p.n_input - j * kKeys);
        const int sbuf = g & 1;
        if (!(ok = warp_mbar_wait(smem_u32(&bars.s_full[sbuf]), (g >> 1) & 1, kTimeoutMmaDone, abort)))
          break;
        tc_fence_after();
        float x[kKeys];  // raw scores of this row
        {
          uint32_t sa[32], sb[32];
          tmem_ld32(t_row + kSCol + sbuf * kKeys, sa);
          tmem_ld32(t_row + kSCol + sbuf * kKeys + 32, sb);
          tmem_ld_wait();
#pragma unroll
          for (int k = 0; k < 32; ++k) {
            x[k] = __uint_as_float(sa[k]);
            x[k + 32] = __uint_as_float(sb[k]);
          }
        }
        if (valid < kKeys) {  // ragged last tile: keys past N_input get weight 0
#pragma unroll
          for (int k = 0; k < kKeys; ++k) x[k] = k < valid ? x[k] : -INFINITY;
        }
        // weights 2^(x * scale_log2 - m): one FFMA and one ex2 per score.  The row sum adds
        // the bf16-rounded weights the P.V product uses, so each output row is an exact
        // weighted mean of V (summing the unrounded weights doubles the error when a few keys
        // dominate)
        float lsum;
        uint32_t w[32];  // P of this row: column c holds keys 2c (low half) and 2c + 1
        auto weights = [&](float neg_m) {
          lsum = 0.f;
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const float p0 = ex2_approx(fmaf(x[2 * c], p.scale_log2, neg_m));
            const float p1 = ex2_approx(fmaf(x[2 * c + 1], p.scale_log2, neg_m));
            w[c] = pack_bf16x2(p0, p1);
            if (!kTcSum) lsum += __uint_as_float(w[c] << 16) + __uint_as_float(w[c] & 0xffff0000u);
          }
        };
        // row maximum of the raw scores (the scale is positive), four independent chains
        auto row_max = [&]() {
          float mx[4];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            mx[c] = x[16 * c];
#pragma unroll
            for (int k = 1; k < 15; k += 2) mx[c] = fmax3(mx[c], x[16 * c + k], x[16 * c + k + 1]);
            mx[c] = fmaxf(mx[c], x[16 * c + 15]);
          }
          return fmaxf(fmax3(mx[0], mx[1], mx[2]), mx[3]) * p.scale_log2;
        };
        float alpha = 1.f;
        if (j == 0) {
          m_run = row_max();
          weights(-m_run);
        } else {
          // The running maximum changes only when a tile exceeds it by 2^kRescaleLog2 (lazy
          // rescale), so the weights are computed against m_run while the tile maximum is
          // found alongside: the ex2 stream does not wait for the maximum.  A tile that does
          // exceed it (rare once a few tiles are in) recomputes its weights below.
          weights(-m_run);
          const float tmax = row_max();
          if (tmax > m_run + kRescaleLog2) {
            alpha = ex2_approx(m_run - tmax);
            m_run = tmax;
          }
        }
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
          // rescaling O needs every earlier P V complete: the last one is tile g - 1
          if (!(ok = warp_mbar_wait(smem_u32(&bars.pv_done), (g - 1) & 1, kTimeoutMmaDone, abort)))
            break;
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < kDh / 32; ++c) {
            uint32_t o[32];
            tmem_ld32(t_row + kOCol + c * 32, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(t_row + kOCol + c * 32, o);
          }
          if (kTcSum) {  // the row-sum columns scale with O
            uint32_t o[16];
            tmem_ld16(t_row + kOCol + kDh, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st16(t_row + kOCol + kDh, o);
          }
          tmem_st_wait();
          weights(-m_run);  // lanes whose maximum did not move recompute the same weights
        }
        tmem_st32(t_row + kSCol + sbuf * kKeys, w);
        tmem_st_wait();
        l_run = l_run * alpha + lsum;
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&bars.p_full[sbuf]));
      }
      // ---- epilogue: O / l -> bf16 -> this warp's staging slots (32 rows x 32 columns, rows
      // of 64 bytes in the 64-byte swizzle: 16-byte chunk k of row r at k ^ ((r >> 1) & 3),
      // bank-conflict free) -> one TMA store per chunk, which clips rows past N_latent and
      // runs while the warp goes on to the next item.  Reading O precedes the next item's
      // first P V, which waits for this warp's next p_full arrival.
      if (!ok || !(ok = warp_mbar_wait(smem_u32(&bars.o_done), it & 1, kTimeoutMmaDone, abort))) break;
      tc_fence_after();
      float l_tot = l_run;
      if (kTcSum) {
        uint32_t lr[16];
        tmem_ld16(t_row + kOCol + kDh, lr);
        tmem_ld_wait();
        l_tot = __uint_as_float(lr[0]);
      }
      const float inv = 1.f / l_tot;
      const int y0 = wi.row0 + quad * 32;  // this warp's first output row
      const bool rows_in = y0 < p.n_latent;
      if (lane == 0) bulk_wait_group_read<0>();  // the previous item's stores read their slots
      __syncwarp();
      // chunks in groups of kSlots (one group unless d = 128): the TMEM load of chunk c + 1
      // is in flight while chunk c is packed; one proxy fence and one bulk group per group
      uint32_t oa[32], ob[32];
      tmem_ld32(t_row + kOCol, oa);
#pragma unroll
      for (int c = 0; c < L::kChunks; ++c) {
        const int slot = c % L::kSlots;
        if (c >= L::kSlots && slot == 0) {  // group reuses the slots: earlier stores read them
          if (lane == 0) bulk_wait_group_read<0>();
          __syncwarp();
        }
        tmem_ld_wait();
        uint32_t* o = (c & 1) ? ob : oa;
        if (c + 1 < L::kChunks) tmem_ld32(t_row + kOCol + (c + 1) * 32, (c & 1) ? oa : ob);
        const uint32_t sbase = staging + (quad * L::kSlots + slot) * L::kChunkBytes;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          st_shared_v4(sbase + lane * 64 + ((k ^ ((lane >> 1) & 3)) << 4),
                       pack_bf16x2(__uint_as_float(o[8 * k + 0]) * inv, __uint_as_float(o[8 * k + 1]) * inv),
                       pack_bf16x2(__uint_as_float(o[8 * k + 2]) * inv, __uint_as_float(o[8 * k + 3]) * inv),
                       pack_bf16x2(__uint_as_float(o[8 * k + 4]) * inv, __uint_as_float(o[8 * k + 5]) * inv),
                       pack_bf16x2(__uint_as_float(o[8 * k + 6]) * inv, __uint_as_float(o[8 * k + 7]) * inv));
        if (slot == L::kSlots - 1 || c == L::kChunks - 1) {  // group complete: store it
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && rows_in) {
            for (int cc = c - slot; cc <= c; ++cc)
              tma_store_3d(&p.to, staging + (quad * L::kSlots + cc % L::kSlots) * L::kChunkBytes,
                           wi.col0 + cc * 32, y0, wi.b);
            bulk_commit_group();
          }
        }
      }
      tc_fence_before();
    }
    if (lane == 0) bulk_wait_group_all();  // stores done before the CTA's shared memory goes
  }

  tc_fence_before();
  __syncthreads();
  if (abort_flag) {  // stable here: every give_up preceded the barrier
    settle_after_give_up();
    __syncthreads();
  }
  tc_fence_after();
  if (threadIdx.x == 0) XATTN_TRACE_POINT(13, 0);
  if (warp == 0) tmem_dealloc(tmem, kTmemCols);
}

}  // namespace mha
}  // namespace xattn
