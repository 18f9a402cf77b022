// Fused fp32-API cross attention for sm_100a: O = softmax(Q K^T / sqrt(D)) V.
//
// Replaces the upstream kernels optimized_cross_attention (kernel_vectorized.cu:17-196),
// tiled/warp/naive (kernel_tiled.cu, kernel_warp_parallel.cu, kernel_naive.cu) and the
// split-K partial (kernel_splitk.cu:42-181).  One kernel family serves all of them.
//
// Shape of the work.  A cluster of two CTAs owns one "row block": 128 query rows of one
// batch, over one key range [k_begin, k_end).  The embedding dimension D is split in two
// halves of Dh = D/2 columns: CTA h owns columns [h*Dh, (h+1)*Dh).  A 128 x D fp32 output
// accumulator (384 KB at D=768) does not fit one SM's 256 KB of tensor memory, while each
// half (128 x 384 fp32 = 384 TMEM columns) does, next to the 128-column score tile.
//
// Per key tile of 128 keys, each CTA:
//   1. S_h = Q[:, half h] . K[tile, half h]^T      tcgen05 kind::tf32, SS, M=128 N=128,
//      streaming 32-column chunks of Q and K through a TMA/mbarrier ring;
//   2. softmax warps copy S_h out of tensor memory (which frees it for the next tile's
//      Q.K^T) and send it to the peer CTA with st.async (distributed shared memory);
//      S = S_0 + S_1 is formed in both CTAs (identical bits: fp32 addition commutes);
//   3. online softmax in the log2 domain (scale log2(e)/sqrt(D) folded into one multiply)
//      with lazy rescaling of O only when the running max grows by more than 2^8; P is
//      rounded to tf32 and written, in place of the received scores, into shared memory
//      in the UMMA K-major layout;
//   4. O_h += P . V[tile, half h]                    tcgen05 kind::tf32, SS, B = V
//      streamed in 16-key chunks, MN-major 128B swizzle with 32-byte atoms.
// The MMA warp issues Q.K^T of tile j+1 before it waits for P of tile j, so the score
// exchange and the softmax of one tile overlap the tensor-core work of the next.  Scores
// never leave the chip.  After the last tile the epilogue divides by the row sum and
// stores fp32 rows, or (split mode) stores the unnormalised partial (m, l, O) triple in
// the upstream split-K scratch layout (kernel_splitk.cu:57: pidx = (b*Nl+row)*S+split).
//
// TF32 truncation bias.  kind::tf32 drops the low 13 mantissa bits of each fp32 operand
// (truncation, measured on B200), which shrinks every operand by its relative truncation
// error.  Q.K^T comes out scaled by ~(1 - e_Q - e_K) -- a softmax temperature shift that
// dominates the error -- and P.V by ~(1 - e_V), where e_X is the least-squares relative
// truncation of operand X: e = sum(d x) / sum(x x) with d = x - trunc_tf32(x).  By default
// every item measures e_Q (its own query rows), e_K and e_V (its key range) on a sample of
// the inputs (trunc_load / trunc_finish) and scales the scores by (1 + e_Q + e_K) and the
// output by (1 + e_V).  Random fp32 mantissas give e ~ 2^-11 / (2 ln 2) = 3.5e-4 each;
// inputs that are already exact in TF32 (widened bf16 / fp16, small integers) give exactly
// e = 0, so they are computed without any compensation.
//
// Warp roles (64 + 128 * kGroups threads): warp 0 = TMA producer, warp 1 = MMA issuer,
// warps 2.. = softmax / exchange / epilogue.  Softmax warp w reads TMEM lanes
// 32*(w%4)..+31 (one query row per thread) and column group (w-2)/4 of the score tile, so
// each thread keeps its 64 scores in registers; row maxima and sums are combined across
// the groups through shared memory.  Every mbarrier wait is bounded (sm100.cuh).
#pragma once

#include "sm100.cuh"

namespace xattn {
namespace fused {

constexpr int kRows = 128;          // query rows per CTA (UMMA M)
constexpr int kKeys = 128;          // keys per tile (UMMA N of Q.K^T)
constexpr int kChunk = 32;          // fp32 columns per 128-byte swizzle row
constexpr int kVKeys = 16;          // keys per V chunk
constexpr int kStageBytes = 32768;  // Q chunk (16 KB) + K chunk (16 KB), or one V chunk
constexpr int kStages = 3;
constexpr int kGroups = 2;                   // softmax column groups per TMEM lane quadrant
constexpr int kGroupCols = kKeys / kGroups;  // score columns per softmax thread
constexpr int kSoftmaxThreads = 128 * kGroups;
constexpr int kSCol = 384;          // TMEM column of the S tile
constexpr int kTmemCols = 512;
constexpr int kXBytes = kRows * kKeys * 4;  // one exchange / P buffer: a 128x128 fp32 tile
constexpr int kXBufs = 2;                   // double-buffered across key tiles
constexpr int kMaxDh = 384;                 // D <= 768
// Warps: 0 producer, 1 MMA issuer, 2..9 softmax, 10.. further producers (registers are
// allocated per group of four warps, so twelve warps cost the softmax warps nothing).
constexpr int kFirstExtraProducer = 2 + kSoftmaxThreads / 32;
constexpr int kProducers = 3;
constexpr int kThreads = 64 + kSoftmaxThreads + 32 * (kProducers - 1);
// A producer waits for the release of stage i - kStages by parity alone; its previous
// stage, i + kStages - kProducers, already required stage i - kProducers <= i - kStages.
static_assert(kProducers <= kStages, "parity-only stage waits need kProducers <= kStages");
constexpr int kSmemBytes = kStages * kStageBytes + kXBufs * kXBytes + 1024;
constexpr float kRescaleLog2 = 8.0f;        // lazy-rescale threshold (factor 256)
// Static shared memory of the kernel (barriers, reduction arrays, slots), kept in the
// budget check below together with the dynamic ring + exchange buffer.
constexpr int kStaticSmemBytes = 1536;
static_assert(kSmemBytes + kStaticSmemBytes <= 232448, "exceeds 227 KB of shared memory per CTA");
// The epilogue stages O in the ring and exchange buffers: 24 KB per softmax warp.
static_assert(kSoftmaxThreads / 32 * (kMaxDh / 32 / kGroups) * 4096 <= kStages * kStageBytes + kXBufs * kXBytes,
              "output staging exceeds the operand buffers");
static_assert(kGroupCols == 64, "two 32-column register halves per softmax thread");

struct Params {
  CUtensorMap tq;   // Q [B][Nl][D] fp32, box {32, 128, 1}, 128B swizzle
  CUtensorMap tk;   // K [B][Ni][D] fp32, box {32, 128, 1}, 128B swizzle
  CUtensorMap tv;   // V [B][Ni][D] fp32, box {32, 16, 1}, 128B swizzle / 32B atoms
  CUtensorMap tk8;  // K [B][Ni][D], box {one 128-byte row of columns, 8 keys, 1} (pair
                    // kernel: the short remainder of a key range folded into its first tile)
  CUtensorMap to;   // output: out {D, Nl, B} box {32, 32, 1}, or po {D, S, Nl, B} box
                    // {32, 1, 32, 1} in split mode; 128B swizzle
  float* out;       // [B][Nl][D]                      (final mode)
  float* po;        // [B][Nl][S][D]   unnormalised O  (split mode)
  float* pm;        // [B][Nl][S]      row max of the scaled score, natural-log units
  float* pl;        // [B][Nl][S]      sum of exp(score - pm)
  int batch, n_latent, n_input, dim, dh;
  int n_row_blocks;  // ceil(Nl / 128)
  int num_splits;    // S (1 in final mode)
  int split_chunk;   // keys per split (upstream rule: ceil(Ni / S))
  int split_mode;    // 0: normalised output, 1: partial triples
  int n_items;       // work items (persistent kernels loop over them)
  float scale_log2;  // log2(e) / sqrt(D) (times a fixed score compensation in comp_mode 2)
  float out_comp;    // fixed output compensation (1 unless comp_mode 2)
  int comp_mode;     // 1: measure the truncation of the inputs per item (fp32 operands only)
  const float* q;    // the inputs as plain pointers, read by the truncation sampling
  const float* k;
  const float* v;
};

// ------------------------------------------------------------------ truncation compensation
// Sample of one item's inputs, loaded by one softmax thread t in [0, 256): a 16-byte piece
// of its own query row, one of K and one of V at positions spread over the item's key range
// (1024 values of each per CTA).  Positions depend on the item, the row and t only, never on
// the CTA's half of D, so the CTAs that share rows (and exchange scores) measure
// bit-identical factors.
constexpr int kTruncPieces = 1;
struct TruncLoads {
  float4 q[kTruncPieces], k[kTruncPieces], v[kTruncPieces];
};

__device__ __forceinline__ void trunc_load(const Params& p, TruncLoads& s, int b, int qrow, int k_begin,
                                           int k_end, int t) {
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  const int c4 = p.dim / 4;  // 16-byte pieces per row (D % 64 == 0 on this path)
  const int nk = k_end - k_begin;
#pragma unroll
  for (int i = 0; i < kTruncPieces; ++i) {
    const int cq = 4 * static_cast<int>((static_cast<unsigned>(qrow) * 13u + (2u * t + i) * 97u + 5u) % c4);
    s.q[i] = qrow < p.n_latent
                 ? __ldg(reinterpret_cast<const float4*>(p.q + (static_cast<size_t>(b) * p.n_latent + qrow) * p.dim + cq))
                 : zero;
    const int key = k_begin + static_cast<int>((static_cast<long long>(2 * t + i) * nk) >> 9);
    const size_t kr = (static_cast<size_t>(b) * p.n_input + key) * p.dim;
    const int ck = 4 * static_cast<int>((static_cast<unsigned>(t) * 29u + i * 131u + 3u) % c4);
    const int cv = 4 * static_cast<int>((static_cast<unsigned>(t) * 53u + i * 71u + 17u) % c4);
    s.k[i] = nk > 0 ? __ldg(reinterpret_cast<const float4*>(p.k + kr + ck)) : zero;
    s.v[i] = nk > 0 ? __ldg(reinterpret_cast<const float4*>(p.v + kr + cv)) : zero;
  }
}

// sum(d x) and sum(x x) of the four values, d = x - trunc_tf32(x)
__device__ __forceinline__ void trunc_add(const float4& x, float& num, float& den) {
  const float e[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float t = __uint_as_float(__float_as_uint(e[i]) & 0xFFFFE000u);
    num = fmaf(e[i] - t, e[i], num);
    den = fmaf(e[i], e[i], den);
  }
}

// Relative truncation from the sums; 0 when nothing was sampled, and for non-finite sums
// (NaN / Inf inputs, overflowing squares), where no compensation is the safe answer.
__device__ __forceinline__ float trunc_ratio(float num, float den) {
  return fminf(fmaxf(num / den, 0.f), 0.0009765625f);  // fmaxf(NaN, 0) = 0; |d| < 2^-10 |x|
}

// Truncation sums of one item of the four-CTA pair kernel, taken by one warp: one 16-byte
// piece of every fourth of the item's 256 query rows (rows past N_latent skipped), kept
// apart per 128-row half, and 32 pieces each of K and V spread over the key range
// [k_begin, k_end) -- 128 values of each, which pins e to a few percent of itself (the
// compensation's own error is then ~1e-5 of a score).  The sample is deliberately small:
// it reads ahead, into L2, lines of an item that has not started, and at the C3 shape
// (inputs beyond L2) 16 pieces per lane instead of 4 cost ~2 % of the kernel's time.
// s = {sum d x, sum x x} of rows 0..127, of rows 128..255, of K, of V, identical in every
// lane (xor butterfly).  All four loads are issued before any is used.  Positions depend on
// the item only, so the two pairs of a cluster (the two halves of D) compute bit-identical
// sums.
__device__ __forceinline__ int trunc_piece_col(unsigned key, unsigned c4) {
  return 4 * static_cast<int>(__umulhi(key * 0x9E3779B1u, c4));  // hashed 16-byte piece < c4
}
__device__ __forceinline__ void trunc_warp_sample(const Params& p, int b, int row_base, int k_begin,
                                                  int k_end, int lane, float (&s)[8]) {
  const unsigned c4 = static_cast<unsigned>(p.dim / 4);  // 16-byte pieces per row
  const int nk = k_end - k_begin;
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  float4 x[4];
#pragma unroll
  for (int i = 0; i < 2; ++i) {  // query rows row_base + 128 i + 4 lane
    const int row = row_base + kRows * i + 4 * lane;
    x[i] = row < p.n_latent
               ? __ldg(reinterpret_cast<const float4*>(p.q + (static_cast<size_t>(b) * p.n_latent + row) * p.dim +
                                                       trunc_piece_col(static_cast<unsigned>(row), c4)))
               : zero;
  }
  const int key = k_begin + static_cast<int>((static_cast<long long>(lane) * nk) >> 5);
#pragma unroll
  for (int i = 0; i < 2; ++i)  // K, V
    x[2 + i] = nk > 0 ? __ldg(reinterpret_cast<const float4*>((i == 0 ? p.k : p.v) +
                                                              (static_cast<size_t>(b) * p.n_input + key) * p.dim +
                                                              trunc_piece_col(2u * lane + 1u + i, c4)))
                      : zero;
#pragma unroll
  for (int i = 0; i < 8; ++i) s[i] = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) trunc_add(x[i], s[2 * i], s[2 * i + 1]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i] += __shfl_xor_sync(0xffffffffu, s[i], o);
}

// This thread's sums of its sample: {sum d x, sum x x} for Q, K and V.
__device__ __forceinline__ void trunc_fold(const TruncLoads& s, float (&v)[6]) {
#pragma unroll
  for (int i = 0; i < 6; ++i) v[i] = 0.f;
#pragma unroll
  for (int i = 0; i < kTruncPieces; ++i) {
    trunc_add(s.q[i], v[0], v[1]);
    trunc_add(s.k[i], v[2], v[3]);
    trunc_add(s.v[i], v[4], v[5]);
  }
}

// Warp sums of the threads' sums into buf[sw] (a [kWarps][6] array in shared memory).
__device__ __forceinline__ void trunc_publish(float (&v)[6], float (*buf)[6], int sw, int lane) {
  // xor butterfly: every lane ends with bit-identical sums
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int i = 0; i < 6; ++i) v[i] += __shfl_xor_sync(0xffffffffu, v[i], o);
  if (lane == 0)
#pragma unroll
    for (int i = 0; i < 6; ++i) buf[sw][i] = v[i];
}

// Once every softmax warp published into `buf` and a barrier ordered that: the score factor
// (1 + e_Q + e_K) and the output factor (1 + e_V), identical in every thread (same sums,
// same order).  No warp may publish into `buf` again before every thread has read it.
template <int kWarps>
__device__ __forceinline__ void trunc_ratios(const float (*buf)[6], float& score_factor,
                                             float& out_factor) {
  float t[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int w = 0; w < kWarps; ++w)
#pragma unroll
    for (int i = 0; i < 6; ++i) t[i] += buf[w][i];
  score_factor = 1.f + trunc_ratio(t[0], t[1]) + trunc_ratio(t[2], t[3]);
  out_factor = 1.f + trunc_ratio(t[4], t[5]);
}

struct __align__(8) Barriers {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t s_full;   // MMA -> softmax: S tile ready in TMEM
  uint64_t s_free;   // softmax -> MMA: S copied out of TMEM, columns reusable
  uint64_t p_full;   // softmax -> MMA: P (and any O rescale) ready
  uint64_t pv_done[kXBufs];  // MMA -> softmax: P.V of a tile using buffer b complete
  uint64_t o_done;   // MMA -> epilogue: last P.V complete
  uint64_t x_full[kXBufs];  // peer -> me: its partial scores are in my exchange buffer b
  uint64_t x_empty;  // peer -> me: the peer's buffer for my next send may be refilled
  uint64_t drain;    // MMA issuer: everything it issued has completed
};

// Round a non-negative finite fp32 value to TF32 (10 explicit mantissa bits), to nearest with
// ties away from zero: add half the weight of the 13 dropped bits, then clear them (a carry
// into the exponent is the correctly rounded result).  Equal to cvt.rna.tf32.f32 for the
// softmax weights it is used on (0 <= P <= 2^8), but runs on the integer pipe instead of
// the conversion unit, which the exponentials already keep busy.
__device__ __forceinline__ uint32_t f2tf32(float x) {
  return (__float_as_uint(x) + 0x1000u) & 0xFFFFE000u;
}

// Exchange layout of the received partial scores, chunk-major: 16-byte chunk i (keys
// 4i..4i+3) of row r at byte (i * 128 + r) * 16, so a warp's 32 rows write and read one
// contiguous 512-byte span.
__device__ __forceinline__ uint32_t x_offset(int chunk, int row) { return (chunk * kRows + row) * 16; }

// P layout, UMMA K-major with 128-byte swizzle: key group g (32 keys) is a 16 KB block of
// 128 rows x 128 bytes; 16-byte chunk c of row r sits at r*128 + (c ^ (r%8))*16.
__device__ __forceinline__ uint32_t p_offset(int chunk, int row) {
  return (chunk >> 3) * 16384 + row * 128 + (((chunk & 7) ^ (row & 7)) << 4);
}

__device__ __forceinline__ void st_shared_f4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

// Epilogue store of O (the CTA's dh columns in TMEM, rows of this warp's lane quadrant)
// through shared memory: the warp's 32-column chunks c = grp, grp + kGroups, .. are scaled
// and written to its staging boxes (4 KB each: 32 rows of 128 bytes, 16-byte piece k of
// row r at k ^ (r % 8) -- the TMA 128-byte swizzle, bank-conflict free), then one lane
// stores them with TMA (boxes of 32 rows x 32 columns, clipped to N_latent) and waits until
// the boxes have been read, so the staging may be reused.  With fewer staging boxes
// (box_cap) than chunks this repeats in rounds.  One row per thread with 16-byte global
// stores took ~12 us per CTA at C3 (each warp store touching 32 rows).
//   stage_base  this warp's staging (box_cap boxes of 4 KB)
//   y0, rows_in the warp's first output row; whether any of its rows exist
__device__ __forceinline__ void store_o_tma(const CUtensorMap* map, bool split_map, uint32_t stage_base,
                                            int box_cap, uint32_t t_row, int dh, int grp, int lane,
                                            float scale, int col0, int split, int y0, int b,
                                            bool rows_in) {
  const int n = (dh / 32 - grp + kGroups - 1) / kGroups;  // chunks of this warp
  auto put = [&](const uint32_t (&o)[32], int i) {
    const uint32_t box = stage_base + (i % box_cap) * 4096 + lane * 128;
#pragma unroll
    for (int k = 0; k < 8; ++k)
      st_shared_f4(box + ((k ^ (lane & 7)) << 4), __uint_as_float(o[4 * k]) * scale,
                   __uint_as_float(o[4 * k + 1]) * scale, __uint_as_float(o[4 * k + 2]) * scale,
                   __uint_as_float(o[4 * k + 3]) * scale);
  };
  int first = 0;  // first chunk of the current round
  auto flush = [&](int last) {  // store chunks first..last, then free their boxes
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0 && rows_in) {
      for (int i = first; i <= last; ++i) {
        const int x = col0 + (grp + i * kGroups) * 32;
        const uint32_t box = stage_base + (i % box_cap) * 4096;
        if (split_map)
          tma_store_4d(map, box, x, split, y0, b);
        else
          tma_store_3d(map, box, x, y0, b);
      }
      bulk_commit_group();
      bulk_wait_group_read<0>();
    }
    __syncwarp();
    first = last + 1;
  };
  uint32_t oa[32], ob[32];  // the TMEM load of the next chunk overlaps the current one's stores
  if (n > 0) tmem_ld32(t_row + grp * 32, oa);
  for (int i = 0; i < n; i += 2) {
    tmem_ld_wait();
    if (i + 1 < n) tmem_ld32(t_row + (grp + (i + 1) * kGroups) * 32, ob);
    put(oa, i);
    if (i == n - 1 || i % box_cap == box_cap - 1) flush(i);
    if (i + 1 < n) {
      tmem_ld_wait();
      if (i + 2 < n) tmem_ld32(t_row + (grp + (i + 2) * kGroups) * 32, oa);
      put(ob, i + 1);
      if (i + 1 == n - 1 || (i + 1) % box_cap == box_cap - 1) flush(i + 1);
    }
  }
}

__device__ __forceinline__ float4 ld_shared_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// Epilogue store of O without bulk copies: each 32 x 32 chunk (c = grp, grp + kGroups, ..)
// goes TMEM -> registers (one row per lane) -> the warp's 4 KB box of shared memory (the
// same swizzled rows as store_o_tma) -> back into registers as row segments (lane l: row
// 4k + l / 8, 16-byte piece l % 8) -> 16-byte streaming global stores, four whole 128-byte
// row segments per warp instruction.  Nothing waits for a store to be read or to land, so
// the box is reused at once; the bulk-copy epilogue instead waited, per round of boxes, for
// the copies to read shared memory (~5.5 us per CTA for 192 KB at C3, with 16 clusters as
// with 33).
//   dst0        output address of this warp's first row at the CTA's first column
//   row_stride  floats between consecutive output rows
//   rows_valid  rows of this warp that exist (<= 0: none)
//   first_read  a cluster mbarrier that lane 0 arrives on once the first chunk has left
//               TMEM (0: none)
__device__ __forceinline__ void store_o_direct(float* dst0, size_t row_stride, uint32_t box,
                                               uint32_t t_row, int dh, int grp, int lane,
                                               float scale, int rows_valid, uint32_t first_read = 0) {
  const int n = (dh / 32 - grp + kGroups - 1) / kGroups;  // chunks of this warp
  const int q = lane & 7;
  auto put = [&](const uint32_t (&o)[32], int i) {
    const int c = grp + i * kGroups;
    const uint32_t rowp = box + lane * 128;
#pragma unroll
    for (int k = 0; k < 8; ++k)
      st_shared_f4(rowp + ((k ^ (lane & 7)) << 4), __uint_as_float(o[4 * k]) * scale,
                   __uint_as_float(o[4 * k + 1]) * scale, __uint_as_float(o[4 * k + 2]) * scale,
                   __uint_as_float(o[4 * k + 3]) * scale);
    __syncwarp();
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int rr = 4 * k + (lane >> 3);
      const float4 v = ld_shared_f4(box + rr * 128 + ((q ^ (rr & 7)) << 4));
      if (rr < rows_valid)
        __stcs(reinterpret_cast<float4*>(dst0 + rr * row_stride + c * 32 + 4 * q), v);
    }
    __syncwarp();
  };
  for (int i = 0; i < n; ++i) {
    uint32_t o[32];
    tmem_ld32(t_row + (grp + i * kGroups) * 32, o);
    tmem_ld_wait();
    if (i == 0 && first_read != 0) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(first_read);
    }
    put(o, i);
  }
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    fused_tf32_kernel(const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* stages = smem;
  uint8_t* xbuf = smem + kStages * kStageBytes;
  __shared__ Barriers bars;
  __shared__ float red[kGroups][kRows];  // per-group row maxima, then row sums (epilogue)
  __shared__ float tstat[kSoftmaxThreads / 32][6];  // truncation sums per softmax warp
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t h = cluster_ctarank();  // which half of D this CTA owns
  const uint32_t peer = h ^ 1u;

  // ---- work item: (batch, row block, split)
  const int item = blockIdx.x / 2;
  const int split = item % p.num_splits;
  const int rb = (item / p.num_splits) % p.n_row_blocks;
  const int b = item / (p.num_splits * p.n_row_blocks);
  const int row0 = rb * kRows;
  const int k_begin = split * p.split_chunk;
  const int k_end = min(k_begin + p.split_chunk, p.n_input);
  const int n_tiles = k_end > k_begin ? (k_end - k_begin + kKeys - 1) / kKeys : 0;
  const int dh = p.dh;
  const int n_qk_chunks = dh / kChunk;
  const int col0 = static_cast<int>(h) * dh;

  if (threadIdx.x == 0) {
    XATTN_TRACE_POINT(14, 0);
    abort_flag = 0;
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&bars.full[s]), 1);
      mbar_init(smem_u32(&bars.empty[s]), 1);
    }
    mbar_init(smem_u32(&bars.s_full), 1);
    mbar_init(smem_u32(&bars.s_free), kSoftmaxThreads);
    mbar_init(smem_u32(&bars.p_full), kSoftmaxThreads);
    for (int b2 = 0; b2 < kXBufs; ++b2) mbar_init(smem_u32(&bars.pv_done[b2]), 1);
    mbar_init(smem_u32(&bars.o_done), 1);
    for (int b2 = 0; b2 < kXBufs; ++b2) mbar_init(smem_u32(&bars.x_full[b2]), 1);
    mbar_init(smem_u32(&bars.x_empty), kSoftmaxThreads / 32);  // one remote arrival per warp
    mbar_init(smem_u32(&bars.drain), 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(&tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  if (warp == 1 && lane == 0) {
    tma_prefetch_desc(&p.tq);
    tma_prefetch_desc(&p.tk);
    tma_prefetch_desc(&p.tv);
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  volatile int* abort = &abort_flag;

  // Ring order, identical for producer and MMA issuer:
  //   QK(0), then for j = 0..n-1: [QK(j+1) if any], V(j).
  if (warp == 0 || warp >= kFirstExtraProducer) {
    // ================================================================ TMA producers
    // Stage i of the ring sequence goes to producer i % kProducers and slot i % kStages;
    // the slot's use count, hence the empty-barrier parity, follows from i.  One issuing
    // thread sustains only a few million copies per second.
    const int pid = warp == 0 ? 0 : warp - kFirstExtraProducer + 1;
    if (elect_one() && n_tiles > 0) {
      bool ok = true;
      int i = 0;
      auto own = [&](uint32_t bytes) -> bool {
        if (i % kProducers != pid) return false;
        const int slot = i % kStages;
        const uint32_t use = static_cast<uint32_t>(i / kStages);
        if (use > 0 &&
            !(ok = mbar_wait(smem_u32(&bars.empty[slot]), (use - 1) & 1u, kTimeoutStageFree, abort)))
          return false;
        mbar_arrive_expect_tx(smem_u32(&bars.full[slot]), bytes);
        return true;
      };
      auto load_qk = [&](int j) {
        const int key0 = k_begin + j * kKeys;
        if (pid == 0) XATTN_TRACE_POINT(0, j);
        for (int c = 0; c < n_qk_chunks && ok; ++c, ++i) {
          if (!own(kStageBytes)) continue;
          const uint32_t st = smem_u32(stages + (i % kStages) * kStageBytes);
          const uint32_t fb = smem_u32(&bars.full[i % kStages]);
          tma_load_3d(st, &p.tq, fb, col0 + c * kChunk, row0, b);
          tma_load_3d(st + 16384, &p.tk, fb, col0 + c * kChunk, key0, b);
        }
      };
      auto load_v = [&](int j) {
        const int key0 = k_begin + j * kKeys;
        const int valid = min(kKeys, k_end - key0);
        const int n_v = (valid + kVKeys - 1) / kVKeys;
        if (pid == 0) XATTN_TRACE_POINT(1, j);
        for (int v = 0; v < n_v && ok; ++v, ++i) {
          if (!own(n_qk_chunks * kVKeys * 128)) continue;
          // all of this CTA's 32-column slabs of kVKeys keys in one box (slab = dim / 32)
          tma_load_4d(smem_u32(stages + (i % kStages) * kStageBytes), &p.tv,
                      smem_u32(&bars.full[i % kStages]), 0, key0 + v * kVKeys, col0 / kChunk, b);
        }
      };
      load_qk(0);
      for (int j = 0; j < n_tiles && ok; ++j) {
        if (j + 1 < n_tiles) load_qk(j + 1);
        load_v(j);
      }
      // Drain (producer 0): every load issued must land before this CTA may exit.
      if (pid == 0) {
        for (int k = max(0, i - kStages); k < i; ++k)
          mbar_wait(smem_u32(&bars.full[k % kStages]), static_cast<uint32_t>(k / kStages) & 1u,
                    kTimeoutDrain, abort);
      }
    }
  } else if (warp == 1) {
    // ================================================================ MMA issuer
    if (elect_one()) {
      if (n_tiles > 0) {
        int s = 0;
        uint32_t phase = 0;
        bool ok = true;
        const uint32_t t_s = tmem + kSCol;
        auto mma_qk = [&](int j) {
          const int key0 = k_begin + j * kKeys;
          const int valid = min(kKeys, k_end - key0);
          const int n_qk = (valid + 15) & ~15;  // UMMA N: multiple of 16 for M=128
          const uint32_t idesc = instr_desc(2, kRows, n_qk, false, false);
          for (int c = 0; c < n_qk_chunks && ok; ++c) {
            if (!(ok = mbar_wait(smem_u32(&bars.full[s]), phase, kTimeoutTmaFull, abort))) break;
            if (c == 0) XATTN_TRACE_POINT(2, j);
            tc_fence_after();
            const uint32_t st = smem_u32(stages + s * kStageBytes);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t ad = smem_desc(st + kk * 32, 16, 1024, kSw128);
              const uint64_t bd = smem_desc(st + 16384 + kk * 32, 16, 1024, kSw128);
              mma_tf32_ss(t_s, ad, bd, idesc, (c | kk) != 0);
            }
            mma_commit(smem_u32(&bars.empty[s]));
            if (++s == kStages) { s = 0; phase ^= 1u; }
          }
          if (ok) mma_commit(smem_u32(&bars.s_full));
          XATTN_TRACE_POINT(3, j);
        };
        mma_qk(0);
        for (int j = 0; j < n_tiles && ok; ++j) {
          if (j + 1 < n_tiles) {
            // S of tile j must have left tensor memory before Q.K^T of tile j+1 lands there.
            if (!(ok = mbar_wait(smem_u32(&bars.s_free), j & 1, kTimeoutSoftmax, abort))) break;
            tc_fence_after();
            mma_qk(j + 1);
            if (!ok) break;
          }
          if (!(ok = mbar_wait(smem_u32(&bars.p_full), j & 1, kTimeoutSoftmax, abort))) break;
          XATTN_TRACE_POINT(4, j);
          tc_fence_after();
          const int key0 = k_begin + j * kKeys;
          const int valid = min(kKeys, k_end - key0);
          const int n_v = (valid + kVKeys - 1) / kVKeys;
          const uint32_t xb = smem_u32(xbuf + (j & 1) * kXBytes);  // P of tile j
          for (int v = 0; v < n_v; ++v) {
            if (!(ok = mbar_wait(smem_u32(&bars.full[s]), phase, kTimeoutTmaFull, abort))) break;
            tc_fence_after();
            const uint32_t st = smem_u32(stages + s * kStageBytes);
            const int ksteps = min(2, (valid - v * kVKeys + 7) / 8);
            for (int kk = 0; kk < ksteps; ++kk) {
              // A = P, keys 16v + 8kk .. +7: key group (16v)/32, byte offset inside the row
              const int key = v * kVKeys + kk * 8;
              const uint64_t ad = smem_desc(xb + (key >> 5) * 16384 + (key & 31) * 4, 16, 1024, kSw128);
              // O columns [0, 256) and [256, dh): at most two instructions (N <= 256).
              for (int n0 = 0; n0 < dh; n0 += 256) {
                const int nn = min(256, dh - n0);
                const uint64_t bd = smem_desc(st + (n0 / kChunk) * (kVKeys * 128) + kk * 1024,
                                              kVKeys * 128, 512, kSw128Atom32);
                mma_tf32_ss(tmem + n0, ad, bd, instr_desc(2, kRows, nn, false, true),
                            (j | v | kk) != 0);
              }
            }
            mma_commit(smem_u32(&bars.empty[s]));
            if (++s == kStages) { s = 0; phase ^= 1u; }
          }
          if (!ok) break;
          mma_commit(smem_u32(&bars.pv_done[j & 1]));
          XATTN_TRACE_POINT(5, j);
        }
        mma_commit(smem_u32(&bars.o_done));
      }
      mma_commit(smem_u32(&bars.drain));
      mbar_wait(smem_u32(&bars.drain), 0, kTimeoutDrain, abort);
    }
  } else {
    // ================================================================ softmax / epilogue
    const int sw = warp - 2;
    const int quad = warp & 3;
    const int grp = sw >> 2;
    const int row = quad * 32 + lane;
    const int cbase = grp * kGroupCols;
    const int ch0 = cbase / 4;  // first 16-byte score chunk of this thread
    const uint32_t t_row = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const uint32_t peer_x_row0 = mapa_shared(smem_u32(xbuf) + x_offset(0, row), peer);
    const uint32_t peer_x_full0 = mapa_shared(smem_u32(&bars.x_full[0]), peer);
    const uint32_t peer_x_empty = mapa_shared(smem_u32(&bars.x_empty), peer);
    const bool arm_thread = (sw == 0 && lane == 0);

    float m_run = -INFINITY;   // reference max used for P (log2 units, lazily updated)
    float m_true = -INFINITY;  // exact running max (log2 units)
    float l_run = 0.f;         // this group's share of the row sum
    bool ok = true;
    // Score scale and output factor, with the measured truncation compensation: the sample
    // is loaded and published now (its loads overlap the first Q.K^T) and reduced after the
    // first tile's named barrier; scores are scaled only after it (the row maximum is taken
    // on unscaled sums, which scaling by a positive factor keeps in order).
    const bool comp = p.comp_mode == 1 && n_tiles > 0;
    float sl2 = p.scale_log2, oc = p.out_comp;
    if (comp) {
      TruncLoads tl;
      trunc_load(p, tl, b, row0 + row, k_begin, k_end, sw * 32 + lane);
      float sums[6];
      trunc_fold(tl, sums);
      trunc_publish(sums, tstat, sw, lane);
    }
    for (int j = 0; j < n_tiles; ++j) {
      const int key0 = k_begin + j * kKeys;
      const int valid = min(kKeys, k_end - key0);
      // ---- copy S_h out of tensor memory, release the columns to the next Q.K^T
      // After a failed bounded wait a warp keeps iterating with the work skipped (later waits
      // fail at once through the abort flag), so every softmax warp reaches each named
      // barrier equally often and none is left in bar.sync.
      const int xb_i = j & 1;
      uint8_t* xcur = xbuf + xb_i * kXBytes;
      const uint32_t peer_x_row = peer_x_row0 + xb_i * kXBytes;
      const uint32_t peer_x_full = peer_x_full0 + xb_i * 8;
      ok = ok && warp_mbar_wait(smem_u32(&bars.s_full), j & 1, kTimeoutMmaDone, abort);
      uint32_t ra[32], rb[32];
      float gmax = -INFINITY;
      if (ok) {
      if (sw == 0 && lane == 0) XATTN_TRACE_POINT(6, j);
      tc_fence_after();
      tmem_ld32(t_row + kSCol + cbase, ra);
      tmem_ld32(t_row + kSCol + cbase + 32, rb);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(smem_u32(&bars.s_free));
      // ---- send S_h into the peer's buffer (j % 2) once the peer has released it
      if (j >= kXBufs) ok = warp_mbar_wait<true>(smem_u32(&bars.x_empty), j & 1,
                                                      kTimeoutExchange, abort);
      if (ok) {
      if (sw == 0 && lane == 0) XATTN_TRACE_POINT(12, j);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        st_async_v4(peer_x_row + (ch0 + i) * (kRows * 16), peer_x_full, __uint_as_float(ra[4 * i]),
                    __uint_as_float(ra[4 * i + 1]), __uint_as_float(ra[4 * i + 2]),
                    __uint_as_float(ra[4 * i + 3]));
#pragma unroll
      for (int i = 0; i < 8; ++i)
        st_async_v4(peer_x_row + (ch0 + 8 + i) * (kRows * 16), peer_x_full,
                    __uint_as_float(rb[4 * i]), __uint_as_float(rb[4 * i + 1]),
                    __uint_as_float(rb[4 * i + 2]), __uint_as_float(rb[4 * i + 3]));
      if (arm_thread) mbar_arrive_expect_tx(smem_u32(&bars.x_full[xb_i]), kXBytes);
      if (sw == 0 && lane == 0) XATTN_TRACE_POINT(7, j);
      ok = warp_mbar_wait<true>(smem_u32(&bars.x_full[xb_i]), (j >> 1) & 1, kTimeoutPeer,
                                       abort);
      }
      if (ok) {
      if (sw == 0 && lane == 0) XATTN_TRACE_POINT(8, j);
      // ---- full score = own + peer, in log2 units, masked; group row max
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float4 o = *reinterpret_cast<const float4*>(xcur + x_offset(ch0 + i, row));
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
      }
      red[grp][row] = gmax;
      // every received score is read before P overwrites the buffer in another layout
      named_bar_sync(1, kSoftmaxThreads);
      if (sw == 0 && lane == 0) XATTN_TRACE_POINT(9, j);
      float tmax = red[0][row];
#pragma unroll
      for (int g = 1; g < kGroups; ++g) tmax = fmaxf(tmax, red[g][row]);
      // the row maxima are read by both groups before either writes the next tile's
      named_bar_sync(2 + quad, 32 * kGroups);
      if (!ok) continue;
      if (comp && j == 0) {  // every warp published its sample before the barrier above
        float fs, fo;
        trunc_ratios<kSoftmaxThreads / 32>(tstat, fs, fo);
        sl2 *= fs;
        oc *= fo;
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
      // O rescale (rare): O must hold every earlier P.V, so wait for the previous one.
      if (__any_sync(0xffffffffu, alpha != 1.f)) {
        if (!(ok = warp_mbar_wait(smem_u32(&bars.pv_done[(j - 1) & 1]), ((j - 1) >> 1) & 1,
                                  kTimeoutMmaDone, abort)))
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
      // ---- P = 2^(t - m), rounded to tf32, into the buffer as the A operand of P.V
      float lsum = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        uint32_t q4[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint32_t tv = i < 8 ? ra[4 * i + e] : rb[4 * (i - 8) + e];
          q4[e] = f2tf32(ex2_approx(fmaf(__uint_as_float(tv), sl2, -m_run)));
          lsum += __uint_as_float(q4[e]);
        }
        *reinterpret_cast<uint4*>(xcur + p_offset(ch0 + i, row)) =
            make_uint4(q4[0], q4[1], q4[2], q4[3]);
      }
      l_run += lsum;
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(smem_u32(&bars.p_full));
      if (sw == 0 && lane == 0) XATTN_TRACE_POINT(10, j);
      // ---- my buffer (j+1) % 2 held P of tile j-1: once that P.V completed, the peer may
      // send its scores of tile j+1 into it.
      if (j >= 1 && j + 1 < n_tiles) {
        if (!(ok = warp_mbar_wait(smem_u32(&bars.pv_done[(j - 1) & 1]), ((j - 1) >> 1) & 1,
                                  kTimeoutMmaDone, abort)))
          continue;
        if (sw == 0 && lane == 0) XATTN_TRACE_POINT(11, j);
        if (lane == 0) mbar_arrive_remote(peer_x_empty);
      }
    }
    // ---- epilogue
    red[grp][row] = l_run;
    named_bar_sync(2 + quad, 32 * kGroups);
    float l_tot = 0.f;
#pragma unroll
    for (int g = 0; g < kGroups; ++g) l_tot += red[g][row];
    const int grow = row0 + row;
    const bool live = grow < p.n_latent;
    if (ok && n_tiles > 0 &&
        warp_mbar_wait(smem_u32(&bars.o_done), 0, kTimeoutMmaDone, abort)) {
      tc_fence_after();
      float scale;
      if (p.split_mode) {
        // Partials relative to the exact max: O' = O * 2^(m_run - m_true), l' likewise.
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
      // every MMA has completed, so the ring and the exchange buffers (the first 224 KB of
      // dynamic shared memory) are free: 24 KB of staging per softmax warp
      store_o_tma(&p.to, p.split_mode != 0, smem_u32(smem) + sw * (kMaxDh / 32 / kGroups) * 4096,
                  kMaxDh / 32 / kGroups, t_row, dh, grp, lane, scale, col0, split, row0 + quad * 32,
                  b, row0 + quad * 32 < p.n_latent);
    } else if (n_tiles == 0 && p.split_mode && live) {
      // Empty split (upstream kernel_splitk.cu:62-71): m = -FLT_MAX, l = 0, O = 0.
      const size_t pidx = (static_cast<size_t>(b) * p.n_latent + grow) * p.num_splits + split;
      float* dst = p.po + pidx * p.dim + col0;
      for (int c = grp; c < dh; c += kGroups) dst[c] = 0.f;
      if (h == 0 && grp == 0) {
        p.pm[pidx] = -3.4028234663852886e38f;
        p.pl[pidx] = 0.f;
      }
    }
  }

  if (threadIdx.x == 0) XATTN_TRACE_POINT(13, 0);
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the peer may still be writing into this CTA's exchange buffer
  if (abort_flag) settle_after_give_up();  // stable here: every give_up preceded the barrier
  cluster_sync();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, kTmemCols);
}

}  // namespace fused
}  // namespace xattn
