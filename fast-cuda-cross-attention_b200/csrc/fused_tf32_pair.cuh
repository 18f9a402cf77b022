// Fused cross attention on 4-CTA clusters: a cta_group::2 row pair per D half, on fp32
// operands (kind::tf32, the fp32 API) or fp16 operands (kind::f16, the upstream WMMA entries).
//
// Same computation as fused_tf32.cuh (read that file first); this variant changes how one
// SM's share of the work is fed.  A cluster of four CTAs owns 256 query rows of one batch
// (and a key range, in split mode):  rank = 2h + r, where h is the half of D the CTA owns
// (as in the two-CTA kernel) and r the 128-row half.  The two CTAs with the same h form a
// cta_group::2 pair: the pair leader (r = 0) issues every MMA for both, with M = 256 rows;
// the K operand of Q.K^T and the V operand of P.V are split between the pair's shared
// memories (each CTA loads half the keys of K and half the columns of V), so every K/V byte
// is loaded once per 256 queries instead of once per 128.  Per fp32 key tile and CTA that
// is 384 KB of operands (Q 192 + K 96 + V 96) instead of 576 KB (fp16: half).  Scores are
// still exchanged between the two D halves (ranks r and r + 2) through distributed shared
// memory (fp32 partial scores in both variants); P stays per CTA (each CTA supplies its own
// 128 rows of P as the A operand of the pair MMA).
//
// Persistent: one cluster per co-resident slot loops over the items (batch, 256-row block,
// key split); the ring, the MMA issuer's ring position and every per-tile barrier phase
// continue across items on a global tile index, so the next item's operands stream while
// the current item finishes.  The epilogue takes O out of TMEM in 32 x 32 chunks, passes each
// through a 4 KB shared-memory box per warp (in the slot of the item's last exchange piece)
// and writes whole 128-byte row segments with 16-byte stores (fused::store_o_direct).
//
// Pair protocol.  TMA loads of both CTAs complete on the leader's full barrier; the
// leader's commits are multicast to both CTAs (empty, s_full, pv_done, o_done) or to the
// D-peer pair (x_empty); the softmax warps of both CTAs release S and publish P by arrivals
// on the leader's s_free / p_full barriers.  No TMA multicast is used.
//
// Operand ring.  Three producer warps share one ring of five 24 KB stages in the order
// QK(0), then per tile QK(j+1), V(j): a Q/K stage is a 128-byte-wide chunk of the CTA's 128
// Q rows and of its half of the K tile, a V stage one 4-D box of keys x the CTA's V slabs.
// Producer 0 also prefetches into L2 the V of the tile being loaded and each producer the
// next tile's K chunk it will load, so fewer stage round trips wait on DRAM.  With five
// stages the stream keeps up: timing builds that skip every load after an item's first
// tile run within 1-2 % of this kernel, whose pace is the tensor-core instruction stream
// and the item boundaries (epilogue, then the next item's first exchange).
//
// Exchange slots.  The partial scores travel in pieces of half a key tile (one softmax
// group's 64 keys): piece use u = 2 g + group of global tile g lands in slot u % 3 of the
// D-peer, where the peer's softmax then writes P over it.  The pair leader hands a slot back
// to the D-peer pair with a commit multicast to both of its CTAs once the P.V instructions
// that read the piece complete (an arrival on their x_empty barrier, no data), so the next
// tile's second piece waits only for the first half of this tile's P.V.  An item's last
// piece is handed back after its epilogue instead, which stages O in that slot.
//
// Folded remainder.  A key range whose last 1..kFold keys would form a short last tile adds
// them to its first tile: an N = 16 Q.K^T per stage into TMEM columns 0..15 (O's, unused
// until that tile's P.V), an extra exchange piece and an extra V stage (see kFold).
#pragma once

#include <cuda_fp16.h>

#include "fused_tf32.cuh"

namespace xattn {
namespace pair4 {

using fused::f2tf32;
using fused::kChunk;
using fused::kGroupCols;
using fused::kGroups;
using fused::kKeys;
using fused::kRescaleLog2;
using fused::kRows;
using fused::kSCol;
using fused::kSoftmaxThreads;
using fused::kTmemCols;
using fused::kXBytes;
using fused::p_offset;
using fused::Params;
using fused::x_offset;

// Element type of the operands: fp32 (kind::tf32, the fp32 API) or fp16 (kind::f16, the
// upstream WMMA entries with fp16 inputs).  A 128-byte swizzle row holds kCols elements;
// Q/K stages and V stages keep their byte sizes, P (the A operand of P.V) is stored in T.
template <typename T>
struct Elem;
template <>
struct Elem<float> {
  static constexpr int kCols = 32;                // fp32 per 128-byte swizzle row
  static constexpr int kVKeys = 32;               // keys per V stage (four K=8 steps)
  static constexpr int kKStep = 8;                // MMA K per instruction
  static constexpr uint32_t kFmt = 2;             // instruction descriptor: tf32
  static constexpr uint32_t kVSwz = kSw128Atom32; // V MN-major: 128-byte swizzle, 32-byte atoms
  static constexpr uint32_t kVSbo = 512;
  // P.V instructions per K step (pair N = dh / n <= 256, whole 32-column slabs per CTA)
  __host__ __device__ static constexpr int n_instr(int dh) { return dh <= 256 ? 1 : 2; }
  __host__ __device__ static constexpr bool supports(int dh) {
    return dh == 64 || dh == 128 || dh == 192 || dh == 256 || dh == 384;
  }
};
template <>
struct Elem<__half> {
  static constexpr int kCols = 64;                // fp16 per 128-byte swizzle row
  static constexpr int kVKeys = 64;               // keys per V stage (four K=16 steps)
  static constexpr int kKStep = 16;
  static constexpr uint32_t kFmt = 0;             // instruction descriptor: f16
  static constexpr uint32_t kVSwz = kSw128;       // V MN-major, 128-byte swizzle
  static constexpr uint32_t kVSbo = 1024;
  // pair N = 128 per instruction: one 64-column slab per CTA
  __host__ __device__ static constexpr int n_instr(int dh) { return dh / 128; }
  __host__ __device__ static constexpr bool supports(int dh) {
    return dh == 128 || dh == 256 || dh == 384;
  }
};

template <typename T>
__device__ __forceinline__ void mma_pair(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t acc) {
  if constexpr (sizeof(T) == 4)
    mma_tf32_ss_pair(d, a, b, idesc, acc);
  else
    mma_f16_ss_pair(d, a, b, idesc, acc);
}
constexpr int kStageBytes = 24576;   // Q chunk 16 KB + K half 8 KB, or a V chunk
// Exchange / P pieces: half a key tile each (one softmax group's 64 keys x 128 rows, fp32,
// 32 KB) in a ring of three slots.  Piece use u = 2 g + group of global tile g goes to slot
// u % 3; the D-peer may send use u once use u - 3 of the slot was consumed by P.V.  Three
// half-tile slots keep the next tile's exchange overlapping this tile's P.V (its second
// piece waits only for the first half of P.V) in 96 KB instead of two whole-tile buffers'
// 128 KB, which leaves room for a fifth ring stage.
constexpr int kPieceBytes = kXBytes / kGroups;
constexpr int kXSlots = 3;
constexpr int kStages = 5;
// Warps: 0 producer, 1 MMA issuer, 2..9 softmax, 10.. further producers.  Registers are
// allocated per group of four warps, so twelve warps cost the softmax warps nothing.
constexpr int kFirstExtraProducer = 2 + kSoftmaxThreads / 32;
constexpr int kProducers = 3;
constexpr int kThreads = 64 + kSoftmaxThreads + 32 * (kProducers - 1);
// A producer waits for the release of stage i - kStages by parity alone.  That parity cannot
// alias an older phase because the producer's previous stage, i + kStages - kProducers,
// already required stage i - kProducers <= i - kStages to be consumed.
static_assert(kProducers <= kStages, "parity-only empty waits need kProducers <= kStages");
constexpr int kXRegion = kXSlots * kPieceBytes;
// Folded remainder: a key range whose last 1..kFold keys would form a short last tile (the
// 16 keys of N_input = 784) adds them to its first tile instead: an N = 16 Q.K^T into TMEM
// columns 0..15 (O's columns, free until that tile's P.V), an extra exchange piece (8 KB
// of a slot) and an extra V stage.  A short tile costs a whole pass over Q.
constexpr int kFold = 16;
constexpr int kKxBytes = 1024;       // per stage: 8 keys x one 128-byte row of the folded K
constexpr int kSmemBytes = kStages * kStageBytes + kXRegion + kStages * kKxBytes + 1024;
constexpr int kStaticSmemBytes = 2048;
static_assert(kSmemBytes + kStaticSmemBytes <= 232448, "exceeds 227 KB of shared memory per CTA");
// Output staging: the exchange slots, split evenly between the softmax warps in 4 KB boxes.
constexpr int kStagePerWarp = kXRegion / (kSoftmaxThreads / 32);
static_assert(kStagePerWarp % 4096 == 0 && kStagePerWarp >= 4096, "output staging boxes");
constexpr int kSoftmaxWarpsPerPair = 2 * kSoftmaxThreads / 32;
// P pieces complete after kSoftmaxWarpsPerPair arrivals: a group's piece by its warps with
// a count of kGroups each, the folded piece (written by every warp) with a count of one
constexpr uint32_t kPieceArrivals = kSoftmaxWarpsPerPair;

// D halves this kernel takes: one pair instruction covers N = dh (dh <= 256) or two of
// N = dh / 2 (dh = 384); each CTA holds N / 2 columns of V per instruction, whole 32-wide
// slabs.
__host__ __device__ constexpr bool supports_dh(int dh) { return Elem<float>::supports(dh); }

struct __align__(8) Barriers {
  uint64_t full[kStages];   // leader: both CTAs' loads of a stage landed
  uint64_t empty[kStages];  // both: the pair MMA consumed a stage (multicast commit)
  uint64_t s_full;          // both: S tile ready (multicast)
  uint64_t s_free;          // leader: both CTAs copied S out of TMEM
  uint64_t p_full[kXSlots];  // leader: both CTAs wrote the P piece in slot b (one barrier per
                             // slot: the pair CTAs are not synchronised between releasing S
                             // and publishing P, so one may publish a later piece first)
  uint64_t pv_done[2];       // both: P.V of tile g complete (barrier g % 2, multicast)
  uint64_t o_done;           // both: last P.V complete (multicast)
  uint64_t x_full[kXSlots];  // D-peer -> me: a partial-score piece landed in my slot b
  uint64_t x_empty[kXSlots]; // the D-peer's slot b may be refilled: one arrival per release,
                             // by the D-peer pair leader's commit after P.V read the piece, or
                             // by the D-peer after an epilogue that staged O in its slots
  uint64_t o_lo_read;        // leader: both CTAs' epilogues read O's first 32 columns (a
                             // folded Q.K^T of the next item writes columns 0..15)
  uint64_t drain;            // leader: its MMAs completed
  uint64_t stats_full[2];    // both: the truncation factors of item k are in tfac[k % 2]
  uint64_t stats_empty[2];   // non-leader: the pair's softmax warps are done with tfac[k % 2]
};

template <typename T>
__global__ void __cluster_dims__(4, 1, 1) __launch_bounds__(kThreads, 1)
    fused_tf32_pair_kernel(const __grid_constant__ Params p) {
  using E = Elem<T>;
  constexpr int kVKeys = E::kVKeys;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* stages = smem;
  uint8_t* xbuf = smem + kStages * kStageBytes;
  uint8_t* kxbuf = xbuf + kXRegion;  // folded K rows, one kKxBytes box per ring slot
  __shared__ Barriers bars;
  __shared__ float red[kGroups][kRows];
  __shared__ __align__(8) float tfac[2][2];  // per item parity: score factor of this CTA's rows, output factor
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  // a split's combine kernel, launched as a programmatic dependent, may take free SM slots
  // now and wait there for this grid's results
  griddep_launch_dependents();
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();
  const uint32_t r = rank & 1u;           // row half (position in the cta_group::2 pair)
  const uint32_t h = rank >> 1;           // D half
  const uint32_t leader = rank & ~1u;     // pair leader
  const uint32_t dpeer = rank ^ 2u;       // same rows, other D half
  const uint16_t pair_mask = static_cast<uint16_t>(3u << leader);
  const bool is_leader = (r == 0);
  // measured TF32 truncation compensation (fp32 operands; fused_tf32.cuh)
  const bool comp = sizeof(T) == 4 && p.comp_mode == 1;

  // ---- work items: (batch, 256-row block, split); the cluster takes items cid,
  // cid + n_clusters, ...  Every role walks the same sequence and numbers the key tiles of
  // its items globally (g): the per-tile barriers' phases follow g, o_done's the item count.
  const int cid = blockIdx.x / 4;
  const int n_clusters = gridDim.x / 4;
  const int n_rb2 = (p.n_latent + 2 * kRows - 1) / (2 * kRows);
  struct Item {
    int b, split, row0, k_begin, k_end, n_tiles;
    int extra;  // keys folded into the first tile (the last `extra` keys of the range)
    __device__ int uses() const { return 2 * n_tiles + (extra > 0); }  // exchange pieces
  };
  auto item_at = [&](int item) {
    Item w;
    w.split = item % p.num_splits;
    const int rb2 = (item / p.num_splits) % n_rb2;
    w.b = item / (p.num_splits * n_rb2);
    w.row0 = rb2 * 2 * kRows + static_cast<int>(r) * kRows;  // this CTA's rows
    w.k_begin = w.split * p.split_chunk;
    w.k_end = min(w.k_begin + p.split_chunk, p.n_input);
    const int nk = w.k_end - w.k_begin;
    w.n_tiles = nk > 0 ? (nk + kKeys - 1) / kKeys : 0;
    w.extra = 0;
    if (nk > kKeys && nk % kKeys != 0 && nk % kKeys <= kFold) {
      w.extra = nk % kKeys;
      --w.n_tiles;
    }
    return w;
  };
  // the cluster's next item with key tiles at or after `item` (p.n_items if none)
  auto with_tiles = [&](int item) {
    while (item < p.n_items && item_at(item).n_tiles == 0) item += n_clusters;
    return item;
  };
  const int dh = p.dh;
  const int n_qk_chunks = dh / E::kCols;
  const int col0 = static_cast<int>(h) * dh;
  const int n_instr = E::n_instr(dh);            // P.V instructions per K step
  const int nn = dh / n_instr;                    // pair N per instruction
  const int spi = nn / (2 * E::kCols);            // V slabs (one swizzle row wide) per CTA per instruction
  const int n_slabs = spi * n_instr;              // V slabs this CTA loads per chunk

  if (threadIdx.x == 0) {
    XATTN_TRACE_POINT(14, 0);
    abort_flag = 0;
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&bars.full[s]), 1);
      mbar_init(smem_u32(&bars.empty[s]), 1);
    }
    mbar_init(smem_u32(&bars.s_full), 1);
    mbar_init(smem_u32(&bars.s_free), kSoftmaxWarpsPerPair);
    for (int i = 0; i < kXSlots; ++i) {
      mbar_init(smem_u32(&bars.p_full[i]), kPieceArrivals);
      mbar_init(smem_u32(&bars.x_full[i]), 1);
      mbar_init(smem_u32(&bars.x_empty[i]), 1);
    }
    for (int i = 0; i < 2; ++i) mbar_init(smem_u32(&bars.pv_done[i]), 1);
    mbar_init(smem_u32(&bars.o_done), 1);
    mbar_init(smem_u32(&bars.o_lo_read), kSoftmaxWarpsPerPair / kGroups);
    mbar_init(smem_u32(&bars.drain), 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&bars.stats_full[i]), 1);
      mbar_init(smem_u32(&bars.stats_empty[i]), kSoftmaxWarpsPerPair);
    }
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc_pair(smem_u32(&tmem_slot), kTmemCols);
    tmem_relinquish_pair();
  }
  if (warp == 1 && lane == 0) {
    tma_prefetch_desc(&p.tq);
    tma_prefetch_desc(&p.tk);
    tma_prefetch_desc(&p.tv);
    tma_prefetch_desc(&p.tk8);
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  volatile int* abort = &abort_flag;
  // Launched as a programmatic dependent: the set-up above (barriers, tensor memory, tensor
  // map prefetch) touches no global memory and overlaps the previous kernel of the stream;
  // nothing below reads inputs or writes outputs before that kernel has completed.
  griddep_wait();

  if (warp == 0 || warp >= kFirstExtraProducer) {
    // ================================================================ TMA producers (both CTAs)
    // kProducers warps share one ring.  The ring's stage sequence is fixed:
    //   QK(0); then for every tile j: QK(j+1) (if any), V(j)
    // and stage index i goes to producer i % kProducers and ring slot i % kStages, so each
    // producer can derive the slot's use count (and the empty-barrier parity to wait for)
    // from i alone.  One issuing warp sustains only a few million copies per second, well
    // short of what the MMAs consume; several issuing warps multiply that rate.
    const int pid = warp == 0 ? 0 : warp - kFirstExtraProducer + 1;
    if (elect_one()) {
      bool ok = true;
      int i = 0;  // stage index in the sequence (continues across items)
      // True if this producer owns stage i and its slot is free; `fb` is then the leader's
      // full barrier of the slot (cluster address), armed for both CTAs' bytes.
      uint32_t fb = 0;
      auto own = [&](uint32_t bytes_per_cta) -> bool {
        if (i % kProducers != pid) return false;
        const int slot = i % kStages;
        const uint32_t use = static_cast<uint32_t>(i / kStages);
        if (use > 0 &&
            !(ok = mbar_wait(smem_u32(&bars.empty[slot]), (use - 1) & 1u, kTimeoutStageFree, abort)))
          return false;
        if (is_leader) mbar_arrive_expect_tx(smem_u32(&bars.full[slot]), 2 * bytes_per_cta);
        fb = mapa_shared(smem_u32(&bars.full[slot]), leader);
        return true;
      };
      for (int item = cid; item < p.n_items && ok; item += n_clusters) {
        const Item w = item_at(item);
        auto load_qk = [&](int j) {
          const int key0 = w.k_begin + j * kKeys;
          const int valid = min(kKeys, w.k_end - key0);
          const int n_qk = (valid + 15) & ~15;
          const int kbase = key0 + static_cast<int>(r) * (n_qk / 2);  // this CTA's half of the keys
          if (pid == 0) {
            XATTN_TRACE_POINT(0, j);
            // warm L2 with this tile's V, loaded about one tile from now (a quarter of the
            // operand reads otherwise miss the near L2 partition)
            for (int v = 0; v * kVKeys < valid; ++v)
              for (int n = 0; n < n_instr; ++n)
                tma_prefetch_4d(&p.tv, 0, key0 + v * kVKeys,
                                (col0 + n * nn + static_cast<int>(r) * (nn / 2)) / E::kCols, w.b);
          }
          const bool fold = j == 0 && w.extra > 0;
          const int xbase = w.k_begin + w.n_tiles * kKeys + static_cast<int>(r) * (kFold / 2);
          for (int c = 0; c < n_qk_chunks && ok; ++c, ++i) {
            if (!own(16384 + 8192 + (fold ? kKxBytes : 0))) continue;
            const uint32_t st = smem_u32(stages + (i % kStages) * kStageBytes);
            tma_load_3d_pair(st, &p.tq, fb, col0 + c * E::kCols, w.row0, w.b);
            tma_load_3d_pair(st + 16384, &p.tk, fb, col0 + c * E::kCols, kbase, w.b);
            if (fold)  // this CTA's half of the folded keys (rows past the range read as zero or are masked)
              tma_load_3d_pair(smem_u32(kxbuf + (i % kStages) * kKxBytes), &p.tk8, fb,
                               col0 + c * E::kCols, xbase, w.b);
            // and the same chunk of the next tile's keys (out-of-range boxes prefetch nothing)
            if (j + 1 < w.n_tiles)
              tma_prefetch_3d(&p.tk, col0 + c * E::kCols, key0 + kKeys + static_cast<int>(r) * (kKeys / 2), w.b);
          }
        };
        auto load_v = [&](int j) {
          const int key0 = w.k_begin + j * kKeys;
          const int valid = min(kKeys, w.k_end - key0);
          const int n_v = (valid + kVKeys - 1) / kVKeys;
          if (pid == 0) XATTN_TRACE_POINT(1, j);
          // the tile's V stages, then (first tile of a folded range) one stage at the folded keys
          const int n_vx = n_v + (j == 0 && w.extra > 0 ? 1 : 0);
          for (int v = 0; v < n_vx && ok; ++v, ++i) {
            if (!own(n_slabs * kVKeys * 128)) continue;
            const uint32_t st = smem_u32(stages + (i % kStages) * kStageBytes);
            const int vkey = v < n_v ? key0 + v * kVKeys : w.k_begin + w.n_tiles * kKeys;
            // one box of spi slabs per instruction: slab index (dim / kCols) is the tensor
            // map's third coordinate
            for (int n = 0; n < n_instr; ++n) {
              const int dim = col0 + n * nn + static_cast<int>(r) * (nn / 2);
              tma_load_4d_pair(st + n * spi * (kVKeys * 128), &p.tv, fb, 0, vkey, dim / E::kCols, w.b);
            }
          }
        };
        if (w.n_tiles == 0) continue;
        load_qk(0);
        for (int j = 0; j < w.n_tiles && ok; ++j) {
          if (j + 1 < w.n_tiles) load_qk(j + 1);
          load_v(j);
        }
      }
      // Drain (producer 0): the pair MMA releases every stage it consumed; wait for the last
      // use of every slot so no load into this CTA's shared memory is still in flight at exit
      // (after a give-up the settle at the end covers them).
      if (pid == 0) {
        for (int k = max(0, i - kStages); k < i; ++k)
          mbar_wait(smem_u32(&bars.empty[k % kStages]), static_cast<uint32_t>(k / kStages) & 1u,
                    kTimeoutDrain, abort);
      }
    }
  } else if (warp == 1) {
    // ================================================================ MMA issuer (pair leader)
    if (is_leader && elect_one()) {
      int s = 0;
      uint32_t phase = 0;
      bool ok = true;
      int g = 0;  // global index of the item's first tile
      int U = 0;  // piece use of the item's first piece
      int n_lo = 0;  // o_lo_read phases waited for
      const uint32_t t_s = tmem + kSCol;
      const uint16_t peer_mask = static_cast<uint16_t>(3u << (leader ^ 2u));  // the D-peer pair
      for (int item = cid; item < p.n_items && ok; item += n_clusters) {
        const Item w = item_at(item);
        if (w.n_tiles == 0) continue;
        auto mma_qk = [&](int j) {
          const int key0 = w.k_begin + j * kKeys;
          const int valid = min(kKeys, w.k_end - key0);
          const int n_qk = (valid + 15) & ~15;
          const uint32_t idesc = instr_desc(E::kFmt, 2 * kRows, n_qk, false, false);
          // folded keys: N = 16 into TMEM columns 0..15, which the previous item's epilogue
          // must have read first
          const bool fold = j == 0 && w.extra > 0;
          const uint32_t idesc_x = instr_desc(E::kFmt, 2 * kRows, kFold, false, false);
          if (fold && g > 0) {
            if (!(ok = mbar_wait<true>(smem_u32(&bars.o_lo_read), static_cast<uint32_t>(n_lo) & 1u,
                                       kTimeoutSoftmax, abort)))
              return;
            ++n_lo;
            tc_fence_after();
          }
          for (int c = 0; c < n_qk_chunks && ok; ++c) {
            if (!(ok = mbar_wait(smem_u32(&bars.full[s]), phase, kTimeoutTmaFull, abort))) break;
            if (c == 0) XATTN_TRACE_POINT(2, j);
            tc_fence_after();
            const uint32_t st = smem_u32(stages + s * kStageBytes);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t ad = smem_desc(st + kk * 32, 16, 1024, kSw128);
              const uint64_t bd = smem_desc(st + 16384 + kk * 32, 16, 1024, kSw128);
              mma_pair<T>(t_s, ad, bd, idesc, (c | kk) != 0);
            }
            if (fold) {
              const uint32_t kx = smem_u32(kxbuf + s * kKxBytes);
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)
                mma_pair<T>(tmem, smem_desc(st + kk * 32, 16, 1024, kSw128),
                            smem_desc(kx + kk * 32, 16, 1024, kSw128), idesc_x, (c | kk) != 0);
            }
            mma_commit_pair_mc(smem_u32(&bars.empty[s]), pair_mask);
            if (++s == kStages) { s = 0; phase ^= 1u; }
          }
          if (ok) mma_commit_pair_mc(smem_u32(&bars.s_full), pair_mask);
          XATTN_TRACE_POINT(3, j);
        };
        // S is single-buffered: the item's first Q.K^T waits until the softmax warps copied
        // the previous item's last S out of TMEM.  (Its first P.V, which overwrites O, waits
        // for P, which the softmax warps publish only after the previous epilogue read O.)
        if (g > 0) {
          if (!(ok = mbar_wait<true>(smem_u32(&bars.s_free), (g - 1) & 1, kTimeoutSoftmax, abort)))
            break;
          tc_fence_after();
        }
        mma_qk(0);
        if (!ok) break;
        const int u_end = U + w.uses();  // one past the item's last piece use
        for (int j = 0; j < w.n_tiles && ok; ++j) {
          const int gj = g + j;
          const bool fold = j == 0 && w.extra > 0;
          const int u0 = U + 2 * j + (j > 0 && w.extra > 0 ? 1 : 0);  // the tile's first piece
          if (j + 1 < w.n_tiles) {
            if (!(ok = mbar_wait<true>(smem_u32(&bars.s_free), gj & 1, kTimeoutSoftmax, abort))) break;
            tc_fence_after();
            mma_qk(j + 1);
            if (!ok) break;
          }
          const int key0 = w.k_begin + j * kKeys;
          const int valid = min(kKeys, w.k_end - key0);
          const int n_v = (valid + kVKeys - 1) / kVKeys;
          const uint32_t idesc_pv = instr_desc(E::kFmt, 2 * kRows, nn, false, true);
          // P pieces of this tile: uses u0 (keys 0..63), u0 + 1 (64..127) and, for the first
          // tile of a folded range, u0 + 2 (the folded keys).  Each is waited for before its
          // first V stage (all of them always, so every slot phase is consumed) and handed
          // back to the D-peer pair by a commit once the P.V instructions reading it complete
          // -- except the item's last piece, whose slot stages the epilogue's output and is
          // handed back after it.
          int pc_ready = -1;
          auto take_piece = [&](int pc) -> bool {
            const int u = u0 + pc;
            if (!mbar_wait<true>(smem_u32(&bars.p_full[u % kXSlots]), static_cast<uint32_t>(u / kXSlots) & 1u,
                                 kTimeoutSoftmax, abort))
              return false;
            tc_fence_after();
            pc_ready = pc;
            return true;
          };
          auto give_piece = [&](int pc) {
            const int u = u0 + pc;
            if (u != u_end - 1) mma_commit_pair_mc(smem_u32(&bars.x_empty[u % kXSlots]), peer_mask);
          };
          if (!(ok = take_piece(0))) break;
          XATTN_TRACE_POINT(4, j);
          for (int v = 0; v < n_v; ++v) {
            const int pc = v * kVKeys / kGroupCols;  // piece of this stage's keys
            if (pc > pc_ready && !(ok = take_piece(pc))) break;
            if (!(ok = mbar_wait(smem_u32(&bars.full[s]), phase, kTimeoutTmaFull, abort))) break;
            tc_fence_after();
            const uint32_t st = smem_u32(stages + s * kStageBytes);
            const uint32_t xb = smem_u32(xbuf) + ((u0 + pc) % kXSlots) * kPieceBytes;
            const int ksteps = min(kVKeys / E::kKStep, (valid - v * kVKeys + E::kKStep - 1) / E::kKStep);
            for (int kk = 0; kk < ksteps; ++kk) {
              const int key = v * kVKeys + kk * E::kKStep - pc * kGroupCols;  // key within the piece
              // P: K-major, kCols keys per 128-byte row, 16 KB per key group
              const uint64_t ad = smem_desc(xb + (key / E::kCols) * 16384 + (key % E::kCols) * sizeof(T),
                                            16, 1024, kSw128);
              for (int n = 0; n < n_instr; ++n) {
                const uint64_t bd = smem_desc(st + n * spi * (kVKeys * 128) + kk * E::kKStep * 128,
                                              kVKeys * 128, E::kVSbo, E::kVSwz);
                mma_pair<T>(tmem + n * nn, ad, bd, idesc_pv, (j | v | kk) != 0);
              }
            }
            mma_commit_pair_mc(smem_u32(&bars.empty[s]), pair_mask);
            if (++s == kStages) { s = 0; phase ^= 1u; }
            if (v == n_v - 1 || (v + 1) * kVKeys % kGroupCols == 0) give_piece(pc);
          }
          if (!ok) break;
          // a piece without valid keys (short last tile) still completes its phases
          for (int pc = pc_ready + 1; pc < kGroups && ok; ++pc)
            if ((ok = take_piece(pc))) give_piece(pc);
          if (!ok) break;
          if (fold) {
            // the folded keys: P piece u0 + 2 (P at 16 KB into its slot), one V stage
            if (!(ok = take_piece(kGroups))) break;
            if (!(ok = mbar_wait(smem_u32(&bars.full[s]), phase, kTimeoutTmaFull, abort))) break;
            tc_fence_after();
            const uint32_t st = smem_u32(stages + s * kStageBytes);
            const uint32_t xb = smem_u32(xbuf) + ((u0 + kGroups) % kXSlots) * kPieceBytes + 16384;
            for (int kk = 0; kk * E::kKStep < w.extra; ++kk) {
              const uint64_t ad = smem_desc(xb + kk * E::kKStep * sizeof(T), 16, 1024, kSw128);
              for (int n = 0; n < n_instr; ++n) {
                const uint64_t bd = smem_desc(st + n * spi * (kVKeys * 128) + kk * E::kKStep * 128,
                                              kVKeys * 128, E::kVSbo, E::kVSwz);
                mma_pair<T>(tmem + n * nn, ad, bd, idesc_pv, true);
              }
            }
            mma_commit_pair_mc(smem_u32(&bars.empty[s]), pair_mask);
            if (++s == kStages) { s = 0; phase ^= 1u; }
            give_piece(kGroups);
          }
          mma_commit_pair_mc(smem_u32(&bars.pv_done[gj & 1]), pair_mask);
          XATTN_TRACE_POINT(5, j);
        }
        if (!ok) break;
        mma_commit_pair_mc(smem_u32(&bars.o_done), pair_mask);
        g += w.n_tiles;
        U = u_end;
      }
      mma_commit_pair_mc(smem_u32(&bars.drain), static_cast<uint16_t>(1u << rank));
      mbar_wait(smem_u32(&bars.drain), 0, kTimeoutDrain, abort);
    } else if (!is_leader && comp) {
      // ============================================================ truncation statistics
      // Warp 1 of the pair's second CTA issues nothing, so it measures the inputs' TF32
      // truncation for the items ahead of the softmax warps: per item, the score factor of
      // each 128-row half, 1 + e_Q(half) + e_K, and the output factor 1 + e_V, written to
      // tfac[k % 2] of the leader (first half) and of this CTA (second half) with st.async,
      // whose bytes complete stats_full[k % 2] there (no fence needed).  Buffer k % 2 is
      // refilled once the pair's sixteen softmax warps are done with item k - 2.
      const uint32_t lead_fac = mapa_shared(smem_u32(&tfac[0][0]), leader);
      const uint32_t own_fac = mapa_shared(smem_u32(&tfac[0][0]), rank);
      const uint32_t lead_full = mapa_shared(smem_u32(&bars.stats_full[0]), leader);
      const uint32_t own_full = mapa_shared(smem_u32(&bars.stats_full[0]), rank);
      bool ok = true;
      int k = 0;
      for (int item = with_tiles(cid); item < p.n_items && ok; item = with_tiles(item + n_clusters), ++k) {
        const int buf = k & 1;
        if (k >= 2 &&
            !(ok = warp_mbar_wait(smem_u32(&bars.stats_empty[buf]), static_cast<uint32_t>((k >> 1) - 1) & 1u,
                                  kTimeoutSoftmax, abort)))
          break;
        const Item f = item_at(item);  // f.row0: this CTA's (second) row half
        float sums[8];
        fused::trunc_warp_sample(p, f.b, f.row0 - kRows, f.k_begin, f.k_end, lane, sums);
        const float ek = fused::trunc_ratio(sums[4], sums[5]);
        const float fo = 1.f + fused::trunc_ratio(sums[6], sums[7]);
        if (lane == 0) {
          st_async_v2(lead_fac + buf * 8, lead_full + buf * 8, 1.f + fused::trunc_ratio(sums[0], sums[1]) + ek, fo);
          st_async_v2(own_fac + buf * 8, own_full + buf * 8, 1.f + fused::trunc_ratio(sums[2], sums[3]) + ek, fo);
          mbar_arrive_expect_tx_cluster(lead_full + buf * 8, 8);
          mbar_arrive_expect_tx_cluster(own_full + buf * 8, 8);
        }
        __syncwarp();
      }
    }
  } else {
    // ================================================================ softmax / epilogue (both)
    // warps 2 .. 2 + kSoftmaxThreads / 32 - 1
    const int sw = warp - 2;
    const int quad = warp & 3;
    const int grp = sw >> 2;
    const int row = quad * 32 + lane;
    const int cbase = grp * kGroupCols;
    const uint32_t t_row = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const uint32_t peer_x_row0 = mapa_shared(smem_u32(xbuf) + x_offset(0, row), dpeer);
    const uint32_t peer_x_full0 = mapa_shared(smem_u32(&bars.x_full[0]), dpeer);
    const uint32_t peer_x_empty0 = mapa_shared(smem_u32(&bars.x_empty[0]), dpeer);
    const uint32_t lead_s_free = mapa_shared(smem_u32(&bars.s_free), leader);
    const uint32_t lead_p_full0 = mapa_shared(smem_u32(&bars.p_full[0]), leader);
    const uint32_t lead_o_lo_read = mapa_shared(smem_u32(&bars.o_lo_read), leader);
    const bool arm_thread = ((sw & 3) == 0 && lane == 0);  // one per group

    bool ok = true;
    int g = 0;   // global index of the item's first tile
    int U = 0;   // piece use of the item's first piece
    int it = 0;  // items with tiles done
    // Exchange permissions.  My group sends piece use u = 2 g + grp into the D-peer's slot
    // u % 3.  Uses 0..2 find their slots free; use u >= 3 waits for the release of use u - 3
    // of its slot (phase u / 3 - 1 of x_empty[u % 3]).  Releases come, in use order per
    // slot, from the D-peer pair leader's commit after the P.V that read the piece, or, for
    // the last piece of an item, from the D-peer after that item's epilogue, which stages
    // the output in that piece's slot (the next item's first pieces go to the other two
    // slots, so they cross while the epilogue runs).
    auto x_empty_parity = [&](int u) -> uint32_t { return static_cast<uint32_t>(u / kXSlots - 1) & 1u; };
    // Truncation compensation: the statistics warp has an item's factors ready in
    // tfac[it % 2] long before its first tile needs them; every softmax thread acquires them
    // while the previous item's epilogue waits for its last P.V (the first item's at its
    // first tile).  Scores are scaled only after the first tile's row-maximum barrier (the
    // maximum is taken on unscaled sums, whose order a positive factor keeps), by one FFMA
    // inside the exponent.
    const uint32_t stats_empty0 = mapa_shared(smem_u32(&bars.stats_empty[0]), leader | 1u);
    for (int item = cid; item < p.n_items; item += n_clusters) {
      const Item w = item_at(item);
      const int b = w.b, split = w.split, row0 = w.row0;
      float m_run = -INFINITY;
      float m_true = -INFINITY;
      float l_run = 0.f;
      float sl2 = p.scale_log2;  // this item's score scale (compensated at its first tile)
    for (int j = 0; j < w.n_tiles; ++j) {
      const int gj = g + j;  // global tile index
      const int key0 = w.k_begin + j * kKeys;
      const int valid = min(kKeys, w.k_end - key0);
      // my group's piece of tile gj: use u, slot u % 3, used for the (u / 3)-th time; the
      // first tile of a folded range also exchanges the folded keys as use ux (8 per thread:
      // keys 8 grp .. 8 grp + 7 of the fold, TMEM columns 0..15)
      const bool fold = j == 0 && w.extra > 0;
      const int u = U + 2 * j + (j > 0 && w.extra > 0 ? 1 : 0) + grp;
      const int ux = U + kGroups;
      const int slot = u % kXSlots;
      const uint32_t x_par = static_cast<uint32_t>(u / kXSlots) & 1u;
      uint8_t* xcur = xbuf + slot * kPieceBytes;
      const uint32_t peer_x_row = peer_x_row0 + slot * kPieceBytes;
      const uint32_t peer_x_full = peer_x_full0 + slot * 8;
      // After a failed bounded wait a warp keeps iterating with the work skipped (later waits
      // fail at once through the abort flag), so every softmax warp reaches each named
      // barrier equally often and none is left in bar.sync.
      ok = ok && warp_mbar_wait(smem_u32(&bars.s_full), gj & 1, kTimeoutMmaDone, abort);
      uint32_t ra[32], rb[32], rx[8];
      float gmax = -INFINITY;
      if (ok) {
        if (sw == 0 && lane == 0) XATTN_TRACE_POINT(6, j);
        tc_fence_after();
        tmem_ld32(t_row + kSCol + cbase, ra);
        tmem_ld32(t_row + kSCol + cbase + 32, rb);
        if (fold) tmem_ld8(t_row + 8 * grp, rx);
        tmem_ld_wait();
        if (sw == 0 && lane == 0) XATTN_TRACE_POINT(18, j);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(lead_s_free);
        if (sw == 0 && lane == 0) XATTN_TRACE_POINT(19, j);
      }
      // the D-peer's slot is free for this use once released (u >= 3)
      if (ok && u >= kXSlots)
        ok = warp_mbar_wait<true>(smem_u32(&bars.x_empty[slot]), x_empty_parity(u), kTimeoutExchange, abort);
      if (ok) {
        if (sw == 0 && lane == 0) XATTN_TRACE_POINT(12, j);
#pragma unroll
        for (int i = 0; i < 8; ++i)
          st_async_v4(peer_x_row + i * (kRows * 16), peer_x_full, __uint_as_float(ra[4 * i]),
                      __uint_as_float(ra[4 * i + 1]), __uint_as_float(ra[4 * i + 2]),
                      __uint_as_float(ra[4 * i + 3]));
#pragma unroll
        for (int i = 0; i < 8; ++i)
          st_async_v4(peer_x_row + (8 + i) * (kRows * 16), peer_x_full,
                      __uint_as_float(rb[4 * i]), __uint_as_float(rb[4 * i + 1]),
                      __uint_as_float(rb[4 * i + 2]), __uint_as_float(rb[4 * i + 3]));
        if (arm_thread) mbar_arrive_expect_tx(smem_u32(&bars.x_full[slot]), kPieceBytes);
        if (sw == 0 && lane == 0) XATTN_TRACE_POINT(7, j);
      }
      if (fold && ok) {
        const int sx = ux % kXSlots;
        if (ux >= kXSlots)
          ok = warp_mbar_wait<true>(smem_u32(&bars.x_empty[sx]), x_empty_parity(ux), kTimeoutExchange, abort);
        if (ok) {
          const uint32_t px = peer_x_row0 + sx * kPieceBytes;
#pragma unroll
          for (int k = 0; k < 2; ++k)
            st_async_v4(px + (2 * grp + k) * (kRows * 16), peer_x_full0 + sx * 8, __uint_as_float(rx[4 * k]),
                        __uint_as_float(rx[4 * k + 1]), __uint_as_float(rx[4 * k + 2]),
                        __uint_as_float(rx[4 * k + 3]));
          if (sw == 0 && lane == 0) mbar_arrive_expect_tx(smem_u32(&bars.x_full[sx]), kRows * kFold * 4);
        }
      }
      if (ok) ok = warp_mbar_wait<true>(smem_u32(&bars.x_full[slot]), x_par, kTimeoutPeer, abort);
      if (ok) {
        if (sw == 0 && lane == 0) XATTN_TRACE_POINT(8, j);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float4 o = *reinterpret_cast<const float4*>(xcur + x_offset(i, row));
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int key = cbase + 4 * i + e;
            uint32_t& rv = i < 8 ? ra[4 * i + e] : rb[4 * (i - 8) + e];
            const float add = e == 0 ? o.x : (e == 1 ? o.y : (e == 2 ? o.z : o.w));
            const float t = key < valid ? __uint_as_float(rv) + add : -INFINITY;  // unscaled
            gmax = fmaxf(gmax, t);
            rv = __float_as_uint(t);
          }
        }
      }
      if (fold && ok) {
        const int sx = ux % kXSlots;
        ok = warp_mbar_wait<true>(smem_u32(&bars.x_full[sx]), static_cast<uint32_t>(ux / kXSlots) & 1u,
                                  kTimeoutPeer, abort);
        if (ok) {
          const uint8_t* xx = xbuf + sx * kPieceBytes;
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            const float4 o = *reinterpret_cast<const float4*>(xx + x_offset(2 * grp + k, row));
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float add = e == 0 ? o.x : (e == 1 ? o.y : (e == 2 ? o.z : o.w));
              const float t = 8 * grp + 4 * k + e < w.extra
                                  ? __uint_as_float(rx[4 * k + e]) + add
                                  : -INFINITY;
              gmax = fmaxf(gmax, t);
              rx[4 * k + e] = __float_as_uint(t);
            }
          }
        }
      }
      red[grp][row] = gmax;
      named_bar_sync(1, kSoftmaxThreads);
      if (sw == 0 && lane == 0) XATTN_TRACE_POINT(9, j);
      float tmax = red[0][row];
#pragma unroll
      for (int gg = 1; gg < kGroups; ++gg) tmax = fmaxf(tmax, red[gg][row]);
      named_bar_sync(2 + quad, 32 * kGroups);
      if (!ok) continue;
      if (sw == 0 && lane == 0) XATTN_TRACE_POINT(15, j);
      if (comp && j == 0) {
        if (it == 0 && !(ok = warp_mbar_wait<true>(smem_u32(&bars.stats_full[0]), 0u, kTimeoutSoftmax, abort)))
          continue;
        sl2 = p.scale_log2 * tfac[it & 1][0];
      }
      tmax *= sl2;  // log2 units from here on
      m_true = fmaxf(m_true, tmax);
      float alpha = 1.f;
      if (j == 0) {
        m_run = tmax;
      } else if (tmax > m_run + kRescaleLog2) {
        alpha = ex2_approx(m_run - tmax);
        m_run = tmax;
      }
      if (__any_sync(0xffffffffu, alpha != 1.f)) {
        if (!(ok = warp_mbar_wait(smem_u32(&bars.pv_done[(gj - 1) & 1]),
                                  static_cast<uint32_t>((gj - 1) >> 1) & 1u, kTimeoutMmaDone,
                                  abort)))
          continue;
        tc_fence_after();
        for (int c = grp; c < dh / 32; c += kGroups) {
          uint32_t o[32];
          tmem_ld32(t_row + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(t_row + c * 32, o);
        }
        tmem_st_wait();
      }
      l_run *= alpha;
      float lsum = 0.f;
      if constexpr (sizeof(T) == 4) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          uint32_t q4[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const uint32_t tv = i < 8 ? ra[4 * i + e] : rb[4 * (i - 8) + e];
            q4[e] = f2tf32(ex2_approx(fmaf(__uint_as_float(tv), sl2, -m_run)));
            lsum += __uint_as_float(q4[e]);
          }
          *reinterpret_cast<uint4*>(xcur + p_offset(i, row)) =
              make_uint4(q4[0], q4[1], q4[2], q4[3]);
        }
      } else {
        // fp16 P: this thread's 64 keys are one 128-byte swizzle row of key group grp; the
        // row sum adds the rounded weights the P.V product uses
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint32_t h4[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int k = 8 * c + 2 * e;
            const uint32_t t0 = k < 32 ? ra[k] : rb[k - 32], t1 = k + 1 < 32 ? ra[k + 1] : rb[k + 1 - 32];
            const __half2 hv = __floats2half2_rn(ex2_approx(fmaf(__uint_as_float(t0), sl2, -m_run)),
                                                 ex2_approx(fmaf(__uint_as_float(t1), sl2, -m_run)));
            const float2 back = __half22float2(hv);
            lsum += back.x + back.y;
            h4[e] = *reinterpret_cast<const uint32_t*>(&hv);
          }
          *reinterpret_cast<uint4*>(xcur + row * 128 + ((c ^ (row & 7)) << 4)) =
              make_uint4(h4[0], h4[1], h4[2], h4[3]);
        }
      }
      if (fold) {
        // the folded keys' P, K-major like the main P, 16 KB into the folded piece's slot
        uint8_t* xx = xbuf + (ux % kXSlots) * kPieceBytes + 16384;
        if constexpr (sizeof(T) == 4) {
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            uint32_t q4[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              q4[e] = f2tf32(ex2_approx(fmaf(__uint_as_float(rx[4 * k + e]), sl2, -m_run)));
              lsum += __uint_as_float(q4[e]);
            }
            *reinterpret_cast<uint4*>(xx + p_offset(2 * grp + k, row)) = make_uint4(q4[0], q4[1], q4[2], q4[3]);
          }
        } else {
          uint32_t h4[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const __half2 hv = __floats2half2_rn(ex2_approx(fmaf(__uint_as_float(rx[2 * e]), sl2, -m_run)),
                                                 ex2_approx(fmaf(__uint_as_float(rx[2 * e + 1]), sl2, -m_run)));
            const float2 back = __half22float2(hv);
            lsum += back.x + back.y;
            h4[e] = *reinterpret_cast<const uint32_t*>(&hv);
          }
          *reinterpret_cast<uint4*>(xx + row * 128 + ((grp ^ (row & 7)) << 4)) =
              make_uint4(h4[0], h4[1], h4[2], h4[3]);
        }
      }
      l_run += lsum;
      if (sw == 0 && lane == 0) XATTN_TRACE_POINT(16, j);
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (sw == 0 && lane == 0) XATTN_TRACE_POINT(17, j);
      if (lane == 0) mbar_arrive_remote(lead_p_full0 + slot * 8, kGroups);  // my group's piece
      if (fold && lane == 0) mbar_arrive_remote(lead_p_full0 + (ux % kXSlots) * 8, 1u);
      if (sw == 0 && lane == 0) XATTN_TRACE_POINT(10, j);
    }
    // ---- epilogue of the item
    red[grp][row] = l_run;
    named_bar_sync(2 + quad, 32 * kGroups);
    float l_tot = 0.f;
#pragma unroll
    for (int gg = 0; gg < kGroups; ++gg) l_tot += red[gg][row];
    named_bar_sync(2 + quad, 32 * kGroups);  // red is rewritten by the next tile
    const int grow = row0 + row;
    const bool live = grow < p.n_latent;
    // the next item's truncation factors (acquired now, used at its first tile)
    if (comp && ok && w.n_tiles > 0 && with_tiles(item + n_clusters) < p.n_items)
      ok = warp_mbar_wait<true>(smem_u32(&bars.stats_full[(it + 1) & 1]), static_cast<uint32_t>((it + 1) >> 1) & 1u,
                                kTimeoutSoftmax, abort);
    const bool have_o = ok && w.n_tiles > 0 &&
                        (ok = warp_mbar_wait(smem_u32(&bars.o_done), it & 1, kTimeoutMmaDone, abort));
    if (have_o) {
      if (sw == 0 && lane == 0) XATTN_TRACE_POINT(11, it);
      tc_fence_after();
      // output factor of the item (tfac[it % 2] is refilled only after the arrival below)
      const float oc = comp ? p.out_comp * tfac[it & 1][1] : p.out_comp;
      float scale;
      if (p.split_mode) {
        const float f = ex2_approx(m_run - m_true);
        scale = f * oc;
        const size_t pidx = (static_cast<size_t>(b) * p.n_latent + grow) * p.num_splits + split;
        if (live && h == 0 && grp == 0) {
          p.pm[pidx] = m_true * 0.69314718055994531f;
          p.pl[pidx] = l_tot * f;
        }
      } else {
        scale = oc / l_tot;
      }
      // o_done (a multicast commit after the item's last P.V) means every P.V of the item
      // completed: the slot of the item's last piece, which the D-peer refills only after
      // the release below, stages O, a 4 KB box per softmax warp
      const int y0 = row0 + quad * 32;
      const size_t rs = p.split_mode ? static_cast<size_t>(p.num_splits) * p.dim : p.dim;
      float* dst0 = p.split_mode
                        ? p.po + ((static_cast<size_t>(b) * p.n_latent + y0) * p.num_splits + split) * p.dim + col0
                        : p.out + (static_cast<size_t>(b) * p.n_latent + y0) * p.dim + col0;
      const uint32_t stage = smem_u32(xbuf) + ((U + w.uses() - 1) % kXSlots) * kPieceBytes;
      // a folded first tile of the next item writes TMEM columns 0..15: group 0's warps
      // report when their first chunk (columns 0..31) has left TMEM
      const int nxt = with_tiles(item + n_clusters);
      const bool lo_wait = nxt < p.n_items && item_at(nxt).extra > 0;
      fused::store_o_direct(dst0, rs, stage + sw * 4096, t_row, dh, grp, lane, scale,
                            min(32, p.n_latent - y0), lo_wait && grp == 0 ? lead_o_lo_read : 0u);
      tc_fence_before();
    } else if (w.n_tiles == 0 && p.split_mode && live) {
      const size_t pidx = (static_cast<size_t>(b) * p.n_latent + grow) * p.num_splits + split;
      float* dst = p.po + pidx * p.dim + col0;
      for (int c = grp; c < dh; c += kGroups) dst[c] = 0.f;
      if (h == 0 && grp == 0) {
        p.pm[pidx] = -3.4028234663852886e38f;
        p.pl[pidx] = 0.f;
      }
    }
    if (w.n_tiles > 0) {
      // Every warp has read its staging box back: hand the slot of the item's last piece
      // back to the D-peer (if the cluster has further tiles).
      if (sw == 0 && lane == 0) XATTN_TRACE_POINT(20, it);
      if (with_tiles(item + n_clusters) < p.n_items) {
        named_bar_sync(1, kSoftmaxThreads);
        if (sw == 0 && lane == 0)
          mbar_arrive_remote(peer_x_empty0 + ((U + w.uses() - 1) % kXSlots) * 8);
      }
      if (comp) {  // this warp is done with tfac[it % 2] (both factors were consumed above)
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(stats_empty0 + (it & 1) * 8);
      }
      g += w.n_tiles;
      U += w.uses();
      ++it;
    }
    }
  }

  if (threadIdx.x == 0) XATTN_TRACE_POINT(13, 0);
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no thread of the cluster issues anything after this
  if (abort_flag) settle_after_give_up();  // stable here: every give_up preceded the barrier
  cluster_sync();
  tc_fence_after();
  if (warp == 0) tmem_dealloc_pair(tmem, kTmemCols);
}

}  // namespace pair4
}  // namespace xattn
