// kernels.so: the C ABI declared in include/xattn.h and the host-side dispatch behind it.
//
// Path selection for an fp32 call (Q, K, V, O fp32, row-major, contiguous):
//   * tensor-core path when D is a multiple of 64 in [64, 768] and the four pointers are
//     16-byte aligned (TMA requirement): the persistent four-CTA pair kernel
//     (fused_tf32_pair.cuh) for D in {128, 256, 384, 512, 768}, the two-CTA kernel
//     (fused_tf32.cuh) for the other D; a key split through a library workspace and the
//     LSE combine is added automatically when the row blocks cannot fill the cluster slots;
//   * generic CUDA-core path (simt.cuh) otherwise.
// fp16 calls run the pair kernel on kind::f16 operands for D in {256, 512, 768}, else widen
// to fp32 (exact) for the paths above; bf16 multi-head calls run mha_bf16.cuh.
// There is no host fallback: every path is a GPU kernel.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>
#include <vector>
#include <utility>

#include "accurate.cuh"
#include "fused_tf32.cuh"
#include "fused_tf32_pair.cuh"
#include "mha_bf16.cuh"
#include "peer.cuh"
#include "simt.cuh"
#include "sm100.cuh"
#include "tmap.h"
#include "xattn.h"

namespace xattn {
namespace {

constexpr int kVersion = 10000;  // 1.0.0
constexpr float kLog2e = 1.4426950408889634f;
// Mean relative truncation error of one TF32 operand for log-uniform mantissas:
// 2^-11 * E[1/m], E[1/m] = 1 / (2 ln 2) for m log-uniform on [1, 2).
constexpr double kTf32TruncBias = 0.00048828125 * 0.72134752044448170;

thread_local int t_last_error = XATTN_OK;
std::atomic<int> g_opt_path{0};
std::atomic<int> g_opt_splits{0};
std::atomic<int> g_opt_wait_us{2000000};
std::atomic<int> g_opt_tf32_comp{1};
std::atomic<int> g_opt_kernel{0};  // 0 auto, 1 two-CTA kernel, 2 four-CTA pair kernel
std::atomic<int> g_opt_accurate{0};  // 1: fp32 entries use the 3xTF32 accurate mode

int set_error(int code) {
  t_last_error = code;
  return code;
}

// ------------------------------------------------------------------ per-device state
struct DeviceState {
  bool init = false;
  int sms = 148;
  int pair_slots = 0;  // co-resident 4-CTA clusters of the pair kernel (0: unknown)
  int wait_us = -1;  // value last copied into g_wait_ns on this device
};
std::mutex g_mu;
DeviceState g_dev[64];

// One-time per-device setup: kernel attributes and the device wait bound.
int prepare_device(int* dev_out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return XATTN_ERR_LAUNCH;
  *dev_out = dev;
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceState& st = g_dev[dev];
  if (!st.init) {
    cudaDeviceGetAttribute(&st.sms, cudaDevAttrMultiProcessorCount, dev);
    if (cudaFuncSetAttribute(fused::fused_tf32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             fused::kSmemBytes) != cudaSuccess)
      return XATTN_ERR_LAUNCH;
    if (cudaFuncSetAttribute(pair4::fused_tf32_pair_kernel<float>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             pair4::kSmemBytes) != cudaSuccess ||
        cudaFuncSetAttribute(pair4::fused_tf32_pair_kernel<__half>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             pair4::kSmemBytes) != cudaSuccess)
      return XATTN_ERR_LAUNCH;
    {
      // the persistent pair kernel launches one cluster per co-resident slot (33 on a B200:
      // four-CTA clusters of one CTA per SM cannot use every SM of a GPC)
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(4 * 1024);
      cfg.blockDim = dim3(pair4::kThreads);
      cfg.dynamicSmemBytes = pair4::kSmemBytes;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, reinterpret_cast<const void*>(pair4::fused_tf32_pair_kernel<float>),
                                         &cfg) == cudaSuccess && n > 0)
        st.pair_slots = n;
      else
        cudaGetLastError();  // unknown: one cluster per item
    }
    if (cudaFuncSetAttribute(accurate::gemm3x_kernel<false>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, accurate::kSmemBytes) != cudaSuccess ||
        cudaFuncSetAttribute(accurate::gemm3x_kernel<true>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, accurate::kSmemBytes) != cudaSuccess)
      return XATTN_ERR_LAUNCH;
    for (const void* fn : {reinterpret_cast<const void*>(mha::mha_bf16_kernel<32>),
                           reinterpret_cast<const void*>(mha::mha_bf16_kernel<64>),
                           reinterpret_cast<const void*>(mha::mha_bf16_kernel<96>),
                           reinterpret_cast<const void*>(mha::mha_bf16_kernel<128>)})
      if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, mha::kSmemBytes) !=
          cudaSuccess)
        return XATTN_ERR_LAUNCH;
    st.init = true;
  }
  const int want = g_opt_wait_us.load();
  if (st.wait_us != want) {
    const unsigned long long ns = static_cast<unsigned long long>(want) * 1000ull;
    if (cudaMemcpyToSymbol(g_wait_ns, &ns, sizeof(ns)) != cudaSuccess) return XATTN_ERR_LAUNCH;
    st.wait_us = want;
  }
  return XATTN_OK;
}

int sm_count(int dev) { return g_dev[dev].sms > 0 ? g_dev[dev].sms : 148; }

// Library workspace for automatic key splits: one grow-only buffer per (device, stream).
// Calls that share a stream are ordered by it; different streams get different buffers.
//
// CUDA graphs: a call captured into a graph bakes the stream's buffer address into it, so a
// buffer that captured work used is never freed (a later growth retires it, and retired
// buffers live until the process exits).  A capture on a stream without a large enough
// buffer allocates one with the thread's capture mode relaxed for that cudaMalloc (an
// allocation enqueues no work on the captured stream).  Graph replays share the buffer
// with calls on the stream they were captured on: order them.
struct Workspace {
  void* ptr = nullptr;
  size_t bytes = 0;
  bool captured = false;  // handed to work that a stream capture recorded
};
std::map<std::pair<int, cudaStream_t>, Workspace> g_ws;
std::vector<void*> g_ws_retired;  // outgrown buffers that captured graphs may still read

void* workspace(int dev, cudaStream_t stream, size_t bytes) {
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess) {
    cudaGetLastError();  // e.g. the legacy stream while another thread captures
    return nullptr;
  }
  const bool capturing = cap != cudaStreamCaptureStatusNone;
  std::lock_guard<std::mutex> lk(g_mu);
  Workspace& w = g_ws[{dev, stream}];
  if (w.bytes < bytes) {
    if (w.ptr != nullptr) {
      if (capturing || w.captured) {
        g_ws_retired.push_back(w.ptr);  // no synchronisation is possible (or safe) here
      } else {
        cudaStreamSynchronize(stream);
        cudaFree(w.ptr);
      }
      w = Workspace{};
    }
    const size_t grow = std::max(bytes, static_cast<size_t>(16) << 20);
    cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
    if (capturing) cudaThreadExchangeStreamCaptureMode(&mode);
    const cudaError_t rc = cudaMalloc(&w.ptr, grow);
    if (capturing) cudaThreadExchangeStreamCaptureMode(&mode);  // back to the caller's mode
    if (rc != cudaSuccess) {
      cudaGetLastError();
      w = Workspace{};
      return nullptr;
    }
    w.bytes = grow;
  }
  if (capturing) w.captured = true;
  return w.ptr;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ------------------------------------------------------------------ tensor-core fp32 path
bool tc_fp32_supported(const float* Q, const float* K, const float* V, const float* O, int D) {
  return D >= 64 && D <= 2 * fused::kMaxDh && D % 64 == 0 && aligned16(Q) && aligned16(K) &&
         aligned16(V) && (O == nullptr || aligned16(O));
}

bool make_fp32_maps(fused::Params& p, const float* Q, const float* K, const float* V, int B,
                    int Nl, int Ni, int D, uint32_t k_box = fused::kKeys,
                    uint32_t v_box = fused::kVKeys) {
  const uint64_t dq[3] = {(uint64_t)D, (uint64_t)Nl, (uint64_t)B};
  const uint64_t sq[2] = {(uint64_t)D * 4, (uint64_t)Nl * D * 4};
  const uint64_t dk[3] = {(uint64_t)D, (uint64_t)Ni, (uint64_t)B};
  const uint64_t sk[2] = {(uint64_t)D * 4, (uint64_t)Ni * D * 4};
  const uint32_t bq[3] = {fused::kChunk, fused::kRows, 1};
  const uint32_t bk[3] = {fused::kChunk, k_box, 1};
  const uint32_t bv[3] = {fused::kChunk, v_box, 1};
  return encode_tmap(&p.tq, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, Q, dq, sq, bq,
                     CU_TENSOR_MAP_SWIZZLE_128B) &&
         encode_tmap(&p.tk, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, K, dk, sk, bk,
                     CU_TENSOR_MAP_SWIZZLE_128B) &&
         encode_tmap(&p.tv, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, V, dk, sk, bv,
                     CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
}

// Output map of the fused kernels' TMA-store epilogue: out {D, Nl, B} with boxes of
// 32 columns x 32 rows, or (split mode) the partials po [B][Nl][S][D] as {D, S, Nl, B} with
// boxes {32, 1, 32, 1}; rows past N_latent are clipped by the TMA.
bool make_out_map(fused::Params& p, float* out, float* po, int B, int Nl, int D, int S,
                  int split_mode) {
  if (split_mode) {
    const uint64_t d[4] = {(uint64_t)D, (uint64_t)S, (uint64_t)Nl, (uint64_t)B};
    const uint64_t st[3] = {(uint64_t)D * 4, (uint64_t)S * D * 4, (uint64_t)Nl * S * D * 4};
    const uint32_t box[4] = {fused::kChunk, 1, 32, 1};
    return encode_tmap(&p.to, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, po, d, st, box,
                       CU_TENSOR_MAP_SWIZZLE_128B);
  }
  const uint64_t d[3] = {(uint64_t)D, (uint64_t)Nl, (uint64_t)B};
  const uint64_t st[2] = {(uint64_t)D * 4, (uint64_t)Nl * D * 4};
  const uint32_t box[3] = {fused::kChunk, 32, 1};
  return encode_tmap(&p.to, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, out, d, st, box,
                     CU_TENSOR_MAP_SWIZZLE_128B);
}

// Score scale and TF32 truncation compensation of a launch.  score_scale < 0 means
// 1/sqrt(D).  Option 4 (default 1): the kernels measure the relative truncation of the
// inputs on a sample per item and compensate exactly that (nothing for inputs already exact
// in TF32); 2: the fixed statistical constants for random mantissas, whatever the inputs;
// 0: no compensation.  Known-exact inputs (widened fp16) take none.
void set_scale(fused::Params& p, const float* Q, const float* K, const float* V, int D,
               float score_scale, bool exact_inputs) {
  const double sc = score_scale < 0.f ? 1.0 / std::sqrt(static_cast<double>(D)) : score_scale;
  const int mode = exact_inputs ? 0 : g_opt_tf32_comp.load();
  const bool fixed = mode == 2;
  p.comp_mode = mode == 1 && Q != nullptr ? 1 : 0;
  p.scale_log2 = static_cast<float>(kLog2e * sc * (fixed ? 1.0 + 2.0 * kTf32TruncBias : 1.0));
  p.out_comp = fixed ? static_cast<float>(1.0 + kTf32TruncBias) : 1.f;
  p.q = Q;
  p.k = K;
  p.v = V;
}

// Launch the fused kernel.  split_mode = 0: normalised output `out`; 1: partials.
int launch_fused(const float* Q, const float* K, const float* V, float* out, float* po,
                 float* pm, float* pl, int B, int Nl, int Ni, int D, int num_splits,
                 int split_chunk, int split_mode, cudaStream_t stream, float score_scale = -1.f,
                 bool exact_inputs = false) {
  fused::Params p;
  if (!make_fp32_maps(p, Q, K, V, B, Nl, Ni, D)) return XATTN_ERR_ARG;
  {
    // V as [B][D/32 slabs][Ni keys][32 columns]: one box holds all D/2/32 slabs of a CTA's
    // half for kVKeys keys, so a V stage is one copy
    const uint64_t dv[4] = {(uint64_t)fused::kChunk, (uint64_t)Ni, (uint64_t)D / fused::kChunk,
                            (uint64_t)B};
    const uint64_t sv[3] = {(uint64_t)D * 4, (uint64_t)fused::kChunk * 4, (uint64_t)Ni * D * 4};
    const uint32_t bv[4] = {fused::kChunk, fused::kVKeys, (uint32_t)(D / 2 / fused::kChunk), 1};
    if (!encode_tmap(&p.tv, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, V, dv, sv, bv,
                     CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B))
      return XATTN_ERR_ARG;
  }
  if (!make_out_map(p, out, po, B, Nl, D, num_splits, split_mode)) return XATTN_ERR_ARG;
  p.out = out;
  p.po = po;
  p.pm = pm;
  p.pl = pl;
  p.batch = B;
  p.n_latent = Nl;
  p.n_input = Ni;
  p.dim = D;
  p.dh = D / 2;
  p.n_row_blocks = (Nl + fused::kRows - 1) / fused::kRows;
  p.num_splits = num_splits;
  p.split_chunk = split_chunk;
  p.split_mode = split_mode;
  set_scale(p, Q, K, V, D, score_scale, exact_inputs);
  const long long items = static_cast<long long>(B) * p.n_row_blocks * num_splits;
  if (items * 2 > 0x7fffffffLL) return XATTN_ERR_ARG;
  p.n_items = static_cast<int>(items);
  fused::fused_tf32_kernel<<<static_cast<unsigned>(items * 2), fused::kThreads, fused::kSmemBytes,
                             stream>>>(p);
  return cudaPeekAtLastError() == cudaSuccess ? XATTN_OK : XATTN_ERR_LAUNCH;
}

// Four-CTA pair kernel (fused_tf32_pair.cuh) on fp32 (kind::tf32) or fp16 (kind::f16)
// operands.  split_mode = 0: normalised output `out`; 1: partial triples po / pm / pl over
// num_splits key chunks of split_chunk keys.
template <typename T>
int launch_fused_pair(const T* Q, const T* K, const T* V, float* out, float* po, float* pm,
                      float* pl, int B, int Nl, int Ni, int D, int num_splits, int split_chunk,
                      int split_mode, cudaStream_t stream, float score_scale = -1.f,
                      bool exact_inputs = false) {
  using E = pair4::Elem<T>;
  constexpr CUtensorMapDataType dt =
      sizeof(T) == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  constexpr uint64_t es = sizeof(T);
  const int dh = D / 2;
  if (!E::supports(dh)) return XATTN_ERR_ARG;
  fused::Params p;
  {
    const uint64_t dq[3] = {(uint64_t)D, (uint64_t)Nl, (uint64_t)B};
    const uint64_t sq[2] = {(uint64_t)D * es, (uint64_t)Nl * D * es};
    const uint64_t dk[3] = {(uint64_t)D, (uint64_t)Ni, (uint64_t)B};
    const uint64_t sk[2] = {(uint64_t)D * es, (uint64_t)Ni * D * es};
    const uint32_t bq[3] = {(uint32_t)E::kCols, fused::kRows, 1};
    const uint32_t bk[3] = {(uint32_t)E::kCols, fused::kKeys / 2, 1};
    const uint32_t bk8[3] = {(uint32_t)E::kCols, pair4::kFold / 2, 1};  // folded keys, half per CTA
    // V as [B][D/kCols slabs][Ni keys][kCols columns]: one box holds all the slabs a CTA
    // needs for one P.V instruction (dh / n_instr / 2 columns), so a V stage is one copy
    // per instruction
    const int spi = dh / E::n_instr(dh) / (2 * E::kCols);
    const uint64_t dv[4] = {(uint64_t)E::kCols, (uint64_t)Ni, (uint64_t)D / E::kCols, (uint64_t)B};
    const uint64_t sv[3] = {(uint64_t)D * es, (uint64_t)E::kCols * es, (uint64_t)Ni * D * es};
    const uint32_t bv[4] = {(uint32_t)E::kCols, (uint32_t)E::kVKeys, (uint32_t)spi, 1};
    if (!encode_tmap(&p.tq, dt, 3, Q, dq, sq, bq, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_tmap(&p.tk, dt, 3, K, dk, sk, bk, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_tmap(&p.tk8, dt, 3, K, dk, sk, bk8, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_tmap(&p.tv, dt, 4, V, dv, sv, bv,
                     sizeof(T) == 4 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B))
      return XATTN_ERR_ARG;
  }
  if (!make_out_map(p, out, po, B, Nl, D, num_splits, split_mode)) return XATTN_ERR_ARG;
  p.out = out;
  p.po = po;
  p.pm = pm;
  p.pl = pl;
  p.batch = B;
  p.n_latent = Nl;
  p.n_input = Ni;
  p.dim = D;
  p.dh = dh;
  p.n_row_blocks = (Nl + 2 * fused::kRows - 1) / (2 * fused::kRows);
  p.num_splits = num_splits;
  p.split_chunk = split_chunk;
  p.split_mode = split_mode;
  if constexpr (sizeof(T) == 4)
    set_scale(p, Q, K, V, D, score_scale, exact_inputs);
  else
    set_scale(p, nullptr, nullptr, nullptr, D, score_scale, true);  // fp16 operands are exact
  const long long items = static_cast<long long>(B) * p.n_row_blocks * num_splits;
  if (items * 4 > 0x7fffffffLL) return XATTN_ERR_ARG;
  p.n_items = static_cast<int>(items);
  // persistent: one cluster per co-resident slot, each looping over items
  int dev = 0;
  cudaGetDevice(&dev);
  const int slots = dev >= 0 && dev < 64 ? g_dev[dev].pair_slots : 0;
  const long long clusters = slots > 0 ? std::min<long long>(items, slots) : items;
  // programmatic stream serialization: the kernel's set-up overlaps the previous kernel of
  // the stream, and it waits (griddepcontrol.wait) before touching global memory
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(clusters * 4));
  cfg.blockDim = dim3(pair4::kThreads);
  cfg.dynamicSmemBytes = pair4::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, pair4::fused_tf32_pair_kernel<T>, p) == cudaSuccess ? XATTN_OK
                                                                                  : XATTN_ERR_LAUNCH;
}

int launch_fused_pair(const float* Q, const float* K, const float* V, float* out, int B, int Nl,
                      int Ni, int D, cudaStream_t stream, float score_scale = -1.f,
                      bool exact_inputs = false) {
  return launch_fused_pair<float>(Q, K, V, out, nullptr, nullptr, nullptr, B, Nl, Ni, D, 1, Ni, 0,
                                  stream, score_scale, exact_inputs);
}

// The pair kernel pays off once 256-row blocks fill the four-CTA cluster slots
// (about SMs / 4.5: 33 on a B200 at this shared-memory size).
bool use_pair_kernel(int dev, int B, int Nl, int D) {
  const int sel = g_opt_kernel.load();
  if (sel == 1 || !pair4::supports_dh(D / 2)) return false;
  if (sel == 2) return true;
  const long long items = static_cast<long long>(B) * ((Nl + 255) / 256);
  return items >= sm_count(dev) * 2 / 9;
}

// Key-split plan of the pair kernel: tile-aligned splits so that batch x 256-row blocks x
// splits fills the co-resident cluster slots (one split when the blocks already do).
void plan_pair_splits(int dev, int B, int Nl, int Ni, int* splits_out, int* chunk_out) {
  const long long items = static_cast<long long>(B) * ((Nl + 255) / 256);
  const int n_tiles = (Ni + fused::kKeys - 1) / fused::kKeys;
  const int slots = g_dev[dev].pair_slots > 0 ? g_dev[dev].pair_slots : std::max(1, sm_count(dev) / 4);
  int splits = g_opt_splits.load();
  if (splits <= 0)
    splits = items < slots ? static_cast<int>(std::min<long long>(n_tiles, slots / items)) : 1;
  splits = std::max(1, std::min(splits, std::max(1, n_tiles)));
  const int chunk = (n_tiles + splits - 1) / splits * fused::kKeys;
  *splits_out = splits == 1 ? 1 : (Ni + chunk - 1) / chunk;
  *chunk_out = *splits_out == 1 ? Ni : chunk;
}

// ------------------------------------------------------------------ generic path
template <typename Tin, typename Tout>
int launch_simt(const Tin* Q, const Tin* K, const Tin* V, Tout* out, float* po, float* pm,
                float* pl, int B, int heads, int Nl, int Ni, int dh, int num_splits,
                int split_chunk, int split_mode, float scale_log2, cudaStream_t stream) {
  simt::Args<Tin, Tout> a;
  a.q = Q;
  a.k = K;
  a.v = V;
  a.out = out;
  a.po = po;
  a.pm = pm;
  a.pl = pl;
  const int ld = heads * dh;
  a.q_bs = static_cast<long long>(Nl) * ld;
  a.k_bs = static_cast<long long>(Ni) * ld;
  a.o_bs = static_cast<long long>(Nl) * ld;
  a.ld_q = a.ld_k = a.ld_o = ld;
  a.heads = heads;
  a.dh = dh;
  a.n_latent = Nl;
  a.n_input = Ni;
  a.num_splits = num_splits;
  a.split_chunk = split_chunk;
  a.split_mode = split_mode;
  a.scale_log2 = scale_log2;
  const size_t smem = static_cast<size_t>(simt::kWarps) * 2 * dh * sizeof(float);
  auto kern = simt::attention_kernel<Tin, Tout>;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
          cudaSuccess)
    return XATTN_ERR_ARG;
  dim3 grid((Nl + simt::kWarps - 1) / simt::kWarps, B * heads, num_splits);
  kern<<<grid, simt::kWarps * 32, smem, stream>>>(a);
  return cudaPeekAtLastError() == cudaSuccess ? XATTN_OK : XATTN_ERR_LAUNCH;
}

// pm_out / pl_out non-null: write the merged partial (unnormalised O, M, L) instead.
int launch_combine(const float* po, const float* pm, const float* pl, float* out, long long rows,
                   int D, int num_splits, cudaStream_t stream, float* pm_out = nullptr,
                   float* pl_out = nullptr) {
  if (rows <= 0) return XATTN_OK;
  if (rows > 0x7fffffffLL || num_splits <= 0) return XATTN_ERR_ARG;
  auto kern = pm_out != nullptr ? simt::combine_kernel<float, true> : simt::combine_kernel<float, false>;
  const bool vec = (D & 3) == 0 && (reinterpret_cast<uintptr_t>(po) & 15) == 0;  // as the kernel
  const long long threads = rows * (vec ? (D + 3) / 4 : D);
  const long long blocks = (threads + simt::kCombineThreads - 1) / simt::kCombineThreads;
  if (blocks > 0x7fffffffLL) return XATTN_ERR_ARG;
  // Programmatic stream serialization: the combine's CTAs may launch while the partial
  // kernel still runs (the pair kernel triggers at its start) and wait in griddep_wait()
  // for its results, so the kernel boundary costs no launch latency.  After any other
  // stream operation this is ordinary stream order.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(blocks));
  cfg.blockDim = dim3(simt::kCombineThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t rc = cudaLaunchKernelEx(&cfg, kern, po, pm, pl, out, rows, D, num_splits, D,
                                            pm_out, pl_out);
  return rc == cudaSuccess ? XATTN_OK : XATTN_ERR_LAUNCH;
}

bool bad_sizes(int B, int Nl, int Ni, int D) { return B < 0 || Nl < 0 || Ni < 0 || D <= 0; }

// Upstream semantics for N_input == 0: softmax over no keys gives an empty weight row and
// bmm with an empty V gives zeros (generate_references.py:17-23 evaluated at Ni = 0).
int zero_output(float* O, int B, int Nl, int D, cudaStream_t stream) {
  const size_t bytes = static_cast<size_t>(B) * Nl * D * sizeof(float);
  if (bytes == 0) return XATTN_OK;
  return cudaMemsetAsync(O, 0, bytes, stream) == cudaSuccess ? XATTN_OK : XATTN_ERR_LAUNCH;
}

// Partials of key ranges without keys: (-FLT_MAX, 0, 0) for n (row, split) entries.
int empty_partials(float* po, float* pm, float* pl, long long n, int D, cudaStream_t stream) {
  if (n <= 0) return XATTN_OK;
  const unsigned blocks = static_cast<unsigned>(std::min<long long>((n * D + 255) / 256, 148LL * 8));
  simt::empty_partials_kernel<<<blocks, 256, 0, stream>>>(po, pm, pl, n, D);
  return cudaPeekAtLastError() == cudaSuccess ? XATTN_OK : XATTN_ERR_LAUNCH;
}

// Key-split plan of the automatic fp32 path: one pass when batch * row blocks fill the
// two-CTA cluster slots (SMs / 2), otherwise enough tile-aligned splits to fill them
// (used for the two-CTA kernel; the pair kernel plans with plan_pair_splits).
void plan_splits(int dev, int B, int Nl, int Ni, int path, int* splits_out, int* chunk_out) {
  const int n_rb = (Nl + fused::kRows - 1) / fused::kRows;
  const long long items = static_cast<long long>(B) * n_rb;
  const int n_tiles = (Ni + fused::kKeys - 1) / fused::kKeys;
  const int slots = std::max(1, sm_count(dev) / 2);
  int splits = g_opt_splits.load();
  if (splits <= 0) {
    splits = 1;
    if (path == 0 && items < slots)
      splits = static_cast<int>(std::min<long long>(n_tiles, slots / std::max(1LL, items)));
  }
  splits = std::max(1, std::min(splits, std::max(1, n_tiles)));
  const int tiles_per = (n_tiles + splits - 1) / splits;
  int chunk = std::max(1, tiles_per) * fused::kKeys;
  splits = std::max(1, (Ni + chunk - 1) / chunk);
  if (splits == 1) chunk = Ni;
  *splits_out = splits;
  *chunk_out = chunk;
}

// Tensor-core fp32 attention with automatic key splits.  partial = false: normalised output
// `out`; true: the (m, l, O) triple of all keys into po / pm / pl.  The four-CTA pair kernel
// takes every D it supports (its row pairs share each K/V tile, 384 KB of operands per CTA
// and tile against the two-CTA kernel's 576 KB); key splits fill its cluster slots when the
// 256-row blocks cannot (C4: 2206 -> 1614 us).  option 5 = 1 forces the two-CTA kernel.
int run_fused_auto(int dev, const float* Q, const float* K, const float* V, float* out, float* po,
                   float* pm, float* pl, int B, int Nl, int Ni, int D, bool partial,
                   cudaStream_t stream) {
  const bool pair = g_opt_kernel.load() != 1 && pair4::supports_dh(D / 2) && Ni > 0;
  int splits = 1, chunk = std::max(1, Ni);
  if (Ni > 0) {
    if (pair)
      plan_pair_splits(dev, B, Nl, Ni, &splits, &chunk);
    else
      plan_splits(dev, B, Nl, Ni, g_opt_path.load(), &splits, &chunk);
  }
  if (splits == 1) {
    if (pair)
      return partial ? launch_fused_pair<float>(Q, K, V, nullptr, po, pm, pl, B, Nl, Ni, D, 1, Ni, 1, stream)
                     : launch_fused_pair(Q, K, V, out, B, Nl, Ni, D, stream);
    return partial ? launch_fused(Q, K, V, nullptr, po, pm, pl, B, Nl, Ni, D, 1, chunk, 1, stream)
                   : launch_fused(Q, K, V, out, nullptr, nullptr, nullptr, B, Nl, Ni, D, 1, Ni, 0, stream);
  }
  // Tile-aligned key split through the library workspace, then the log-sum-exp merge.
  const size_t rows = static_cast<size_t>(B) * Nl;
  const size_t po_n = rows * splits * D, ml_n = rows * splits;
  auto r64 = [](size_t n) { return (n + 63) / 64 * 64; };
  float* ws = static_cast<float*>(workspace(dev, stream, (r64(po_n) + 2 * r64(ml_n)) * sizeof(float)));
  if (ws == nullptr) return XATTN_ERR_NOMEM;
  float* wpo = ws;
  float* wpm = wpo + r64(po_n);
  float* wpl = wpm + r64(ml_n);
  const int rc = pair ? launch_fused_pair<float>(Q, K, V, nullptr, wpo, wpm, wpl, B, Nl, Ni, D, splits,
                                                 chunk, 1, stream)
                      : launch_fused(Q, K, V, nullptr, wpo, wpm, wpl, B, Nl, Ni, D, splits, chunk, 1,
                                     stream);
  if (rc != XATTN_OK) return rc;
  return partial ? launch_combine(wpo, wpm, wpl, po, static_cast<long long>(rows), D, splits, stream, pm, pl)
                 : launch_combine(wpo, wpm, wpl, out, static_cast<long long>(rows), D, splits, stream);
}

// The fp32 entry: all four upstream fp32 names and xattn_fp32 land here.
// ------------------------------------------------------------------ 3xTF32 accurate mode
// Batched GEMM launch: C[b] = A[b] (m x k, K-major) x B[b]^T (K-major, n x k) or x B[b]
// (MN-major, k x n).  a_ld / b_ld are row strides in floats; the maps bound rows and K by
// m, n, k, so the TMA zero-fills beyond them whatever the row padding holds.
int launch_gemm3x(const float* A, const float* As, int a_ld, const float* Bm, const float* Bs,
                  int b_ld, bool b_mn_major, float* C, int ldc, int batch, int m, int n, int k,
                  cudaStream_t stream) {
  accurate::GemmParams p;
  const uint64_t da[3] = {(uint64_t)k, (uint64_t)m, (uint64_t)batch};
  const uint64_t sa[2] = {(uint64_t)a_ld * 4, (uint64_t)m * a_ld * 4};
  const uint32_t ba[3] = {accurate::kChunk, accurate::kTile, 1};
  if (!encode_tmap(&p.ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, A, da, sa, ba, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_tmap(&p.tas, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, As, da, sa, ba, CU_TENSOR_MAP_SWIZZLE_128B))
    return XATTN_ERR_ARG;
  if (b_mn_major) {  // B is k x n, rows contiguous along n: {32 columns, k rows, n/32 slabs, batch}
    const uint64_t db[4] = {(uint64_t)accurate::kChunk, (uint64_t)k, (uint64_t)n / accurate::kChunk,
                            (uint64_t)batch};
    const uint64_t sb[3] = {(uint64_t)b_ld * 4, (uint64_t)accurate::kChunk * 4, (uint64_t)k * b_ld * 4};
    const uint32_t bb[4] = {accurate::kChunk, accurate::kChunk, accurate::kTile / accurate::kChunk, 1};
    if (!encode_tmap(&p.tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, Bm, db, sb, bb,
                     CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B) ||
        !encode_tmap(&p.tbs, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, Bs, db, sb, bb,
                     CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B))
      return XATTN_ERR_ARG;
  } else {
    const uint64_t db[3] = {(uint64_t)k, (uint64_t)n, (uint64_t)batch};
    const uint64_t sb[2] = {(uint64_t)b_ld * 4, (uint64_t)n * b_ld * 4};
    if (!encode_tmap(&p.tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, Bm, db, sb, ba, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_tmap(&p.tbs, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, Bs, db, sb, ba, CU_TENSOR_MAP_SWIZZLE_128B))
      return XATTN_ERR_ARG;
  }
  p.c = C;
  p.c_batch_stride = static_cast<long long>(m) * ldc;
  p.ldc = ldc;
  p.m = m;
  p.n = n;
  p.k = k;
  p.tiles_m = (m + accurate::kTile - 1) / accurate::kTile;
  p.tiles_n = (n + accurate::kTile - 1) / accurate::kTile;
  const long long ctas = static_cast<long long>(p.tiles_m) * p.tiles_n * batch;
  if (ctas > 0x7fffffffLL) return XATTN_ERR_ARG;
  if (b_mn_major)
    accurate::gemm3x_kernel<true><<<static_cast<unsigned>(ctas), accurate::kThreads,
                                    accurate::kSmemBytes, stream>>>(p);
  else
    accurate::gemm3x_kernel<false><<<static_cast<unsigned>(ctas), accurate::kThreads,
                                     accurate::kSmemBytes, stream>>>(p);
  return cudaPeekAtLastError() == cudaSuccess ? XATTN_OK : XATTN_ERR_LAUNCH;
}

// fp32 attention in the 3xTF32 accurate mode (accurate.cuh): residuals of Q, K, V; S = Q K^T;
// row softmax into P (+ residual); O = P V.  Workspace: 2 B Nl Ni_pad + B Nl D + 2 B Ni D
// floats (Ni_pad = Ni rounded up to 4, a 16-byte row stride).
int run_fp32_accurate(int dev, const float* Q, const float* K, const float* V, float* O, int B,
                      int Nl, int Ni, int D, cudaStream_t stream) {
  const int ni_pad = (Ni + 3) / 4 * 4;
  const size_t nq = static_cast<size_t>(B) * Nl * D, nk = static_cast<size_t>(B) * Ni * D;
  const size_t ns = static_cast<size_t>(B) * Nl * ni_pad;
  auto r64 = [](size_t n) { return (n + 63) / 64 * 64; };
  float* ws = static_cast<float*>(
      workspace(dev, stream, (r64(nq) + 2 * r64(nk) + 2 * r64(ns)) * sizeof(float)));
  if (ws == nullptr) return XATTN_ERR_NOMEM;
  float* qs = ws;
  float* ks = qs + r64(nq);
  float* vs = ks + r64(nk);
  float* sp = vs + r64(nk);   // S, then P in place
  float* ps = sp + r64(ns);   // residual of P
  const int sms = sm_count(dev);
  for (auto [src, dst, n] : {std::tuple<const float*, float*, size_t>{Q, qs, nq}, {K, ks, nk}, {V, vs, nk}}) {
    const unsigned blocks = static_cast<unsigned>(std::min<long long>((n + 255) / 256, sms * 8LL));
    accurate::split_residual_kernel<<<blocks, 256, 0, stream>>>(src, dst, static_cast<long long>(n));
  }
  if (cudaPeekAtLastError() != cudaSuccess) return XATTN_ERR_LAUNCH;
  int rc = launch_gemm3x(Q, qs, D, K, ks, D, false, sp, ni_pad, B, Nl, Ni, D, stream);
  if (rc != XATTN_OK) return rc;
  const long long rows = static_cast<long long>(B) * Nl;
  accurate::softmax_rows_kernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0, stream>>>(
      sp, ps, rows, Ni, ni_pad, static_cast<float>(1.0 / std::sqrt(static_cast<double>(D))));
  if (cudaPeekAtLastError() != cudaSuccess) return XATTN_ERR_LAUNCH;
  return launch_gemm3x(sp, ps, ni_pad, V, vs, D, true, O, D, B, Nl, D, Ni, stream);
}

int run_fp32(const float* Q, const float* K, const float* V, float* O, int B, int Nl, int Ni,
             int D, cudaStream_t stream) {
  if (bad_sizes(B, Nl, Ni, D)) return set_error(XATTN_ERR_ARG);
  if (B == 0 || Nl == 0) return set_error(XATTN_OK);
  if (O == nullptr) return set_error(XATTN_ERR_ARG);
  if (Ni == 0) return set_error(zero_output(O, B, Nl, D, stream));
  if (Q == nullptr || K == nullptr || V == nullptr) return set_error(XATTN_ERR_ARG);
  int dev = 0;
  int rc = prepare_device(&dev);
  if (rc != XATTN_OK) return set_error(rc);
  const int path = g_opt_path.load();
  const float scale_log2 = kLog2e / std::sqrt(static_cast<float>(D));
  if (g_opt_accurate.load() != 0 && path != 2) {
    // 3xTF32 on the tensor cores where TMA can read the operands; otherwise the generic
    // kernel, which computes in plain fp32 and is as accurate
    if (D % 32 == 0 && aligned16(Q) && aligned16(K) && aligned16(V) && aligned16(O) &&
        static_cast<long long>(B) * Nl < 0x7fffffffLL)
      return set_error(run_fp32_accurate(dev, Q, K, V, O, B, Nl, Ni, D, stream));
    return set_error(launch_simt<float, float>(Q, K, V, O, nullptr, nullptr, nullptr, B, 1, Nl, Ni,
                                               D, 1, Ni, 0, scale_log2, stream));
  }
  if (path == 2 || !tc_fp32_supported(Q, K, V, O, D)) {
    return set_error(launch_simt<float, float>(Q, K, V, O, nullptr, nullptr, nullptr, B, 1, Nl, Ni,
                                               D, 1, Ni, 0, scale_log2, stream));
  }
  return set_error(run_fused_auto(dev, Q, K, V, O, nullptr, nullptr, nullptr, B, Nl, Ni, D, false,
                                  stream));
}

int run_splitk(const float* Q, const float* K, const float* V, float* O, float* po, float* pm,
               float* pl, int B, int Nl, int Ni, int D, int S, cudaStream_t stream) {
  if (bad_sizes(B, Nl, Ni, D) || S <= 0) return set_error(XATTN_ERR_ARG);
  if (B == 0 || Nl == 0) return set_error(XATTN_OK);
  if (O == nullptr || po == nullptr || pm == nullptr || pl == nullptr ||
      (Ni > 0 && (Q == nullptr || K == nullptr || V == nullptr)))  // no keys: K, V unused
    return set_error(XATTN_ERR_ARG);
  int dev = 0;
  int rc = prepare_device(&dev);
  if (rc != XATTN_OK) return set_error(rc);
  if (Ni == 0) {  // every split empty: empty partials, zero output (what the combine gives)
    rc = empty_partials(po, pm, pl, static_cast<long long>(B) * Nl * S, D, stream);
    return set_error(rc != XATTN_OK ? rc : zero_output(O, B, Nl, D, stream));
  }
  const int chunk = std::max(1, (Ni + S - 1) / S);  // kernel_splitk.cu:59
  const float scale_log2 = kLog2e / std::sqrt(static_cast<float>(D));
  if (g_opt_path.load() == 2 || !tc_fp32_supported(Q, K, V, O, D) || !aligned16(po))
    rc = launch_simt<float, float>(Q, K, V, nullptr, po, pm, pl, B, 1, Nl, Ni, D, S, chunk, 1,
                                   scale_log2, stream);
  else if (g_opt_kernel.load() != 1 && pair4::supports_dh(D / 2))
    rc = launch_fused_pair<float>(Q, K, V, nullptr, po, pm, pl, B, Nl, Ni, D, S, chunk, 1, stream);
  else
    rc = launch_fused(Q, K, V, nullptr, po, pm, pl, B, Nl, Ni, D, S, chunk, 1, stream);
  if (rc != XATTN_OK) return set_error(rc);
  return set_error(launch_combine(po, pm, pl, O, static_cast<long long>(B) * Nl, D, S, stream));
}

// fp16 entries (upstream kernel_wmma.cu / kernel_wmma_splitk.cu; Q pre-scaled by 1/sqrt(D)
// on the host, cuda_wrappers.py:635-640), score scale 1.  D in {256, 512, 768}: the pair
// kernel on kind::f16 operands (fp16 products exact in the fp32 accumulator).  Other
// tensor-core D: every fp16 value is exactly representable in TF32, so the inputs are
// widened to fp32 in the library workspace for the TF32 kernels (no truncation
// compensation).  S = 0: the plain entry (automatic kernel and key split); S > 0: the split
// entry, partials into the caller's po/pm/pl with the upstream chunk of
// max(16, round_up(ceil(Ni/S), 16)) keys (kernel_wmma_splitk.cu:52).  Shapes the
// tensor-core kernels do not take run the generic kernel on the fp16 data directly.
int run_half(const __half* Q, const __half* K, const __half* V, float* O, float* po, float* pm,
             float* pl, int B, int Nl, int Ni, int D, int S, cudaStream_t stream) {
  int dev = 0;
  int rc = prepare_device(&dev);
  if (rc != XATTN_OK) return rc;
  const int chunk16 = S > 0 ? std::max(16, ((Ni + S - 1) / S + 15) / 16 * 16) : Ni;
  const bool tc = g_opt_path.load() != 2 && D % 64 == 0 && D >= 64 && D <= 2 * fused::kMaxDh &&
                  aligned16(Q) && aligned16(K) && aligned16(V) && aligned16(O) &&
                  (S == 0 || aligned16(po));
  if (!tc) {
    if (S == 0)
      return launch_simt<__half, float>(Q, K, V, O, nullptr, nullptr, nullptr, B, 1, Nl, Ni, D, 1,
                                        Ni, 0, kLog2e, stream);
    rc = launch_simt<__half, float>(Q, K, V, nullptr, po, pm, pl, B, 1, Nl, Ni, D, S, chunk16, 1,
                                    kLog2e, stream);
    if (rc != XATTN_OK) return rc;
    return launch_combine(po, pm, pl, O, static_cast<long long>(B) * Nl, D, S, stream);
  }
  // Native fp16: the pair kernel on kind::f16 operands (D halves that split into whole
  // 64-column slabs per P.V instruction: D = 256, 512, 768), Q pre-scaled by the caller.
  // Key splits fill the cluster slots when there are fewer 256-row blocks than slots.
  if (pair4::Elem<__half>::supports(D / 2) && g_opt_kernel.load() != 1) {
    const long long rows_all = static_cast<long long>(B) * Nl;
    if (S > 0) {  // upstream split-K entry: caller scratch, chunk rounded up to 16 keys
      rc = launch_fused_pair<__half>(Q, K, V, nullptr, po, pm, pl, B, Nl, Ni, D, S, chunk16, 1,
                                     stream, 1.f, true);
      if (rc != XATTN_OK) return rc;
      return launch_combine(po, pm, pl, O, rows_all, D, S, stream);
    }
    int splits = 1, chunk = Ni;
    plan_pair_splits(dev, B, Nl, Ni, &splits, &chunk);
    if (splits == 1)
      return launch_fused_pair<__half>(Q, K, V, O, nullptr, nullptr, nullptr, B, Nl, Ni, D, 1, Ni,
                                       0, stream, 1.f, true);
    const size_t po_n = static_cast<size_t>(rows_all) * splits * D, ml_n = static_cast<size_t>(rows_all) * splits;
    auto r64 = [](size_t n) { return (n + 63) / 64 * 64; };
    float* ws = static_cast<float*>(workspace(dev, stream, (r64(po_n) + 2 * r64(ml_n)) * sizeof(float)));
    if (ws == nullptr) return XATTN_ERR_NOMEM;
    float* wpo = ws;
    float* wpm = wpo + r64(po_n);
    float* wpl = wpm + r64(ml_n);
    rc = launch_fused_pair<__half>(Q, K, V, nullptr, wpo, wpm, wpl, B, Nl, Ni, D, splits, chunk, 1,
                                   stream, 1.f, true);
    if (rc != XATTN_OK) return rc;
    return launch_combine(wpo, wpm, wpl, O, rows_all, D, splits, stream);
  }
  // plan first, so one workspace request covers the widened inputs and any split partials
  const bool pair = S == 0 && g_opt_splits.load() <= 0 && use_pair_kernel(dev, B, Nl, D);
  int splits = 1, chunk = Ni;
  if (S == 0 && !pair) plan_splits(dev, B, Nl, Ni, g_opt_path.load(), &splits, &chunk);
  const size_t nq = static_cast<size_t>(B) * Nl * D, nk = static_cast<size_t>(B) * Ni * D;
  const size_t rows = static_cast<size_t>(B) * Nl;
  const size_t po_elems = splits > 1 ? rows * splits * D : 0;
  const size_t ml_elems = splits > 1 ? rows * splits : 0;
  // each region rounded to 64 floats (256 B) so every base stays 16-byte aligned
  auto r64 = [](size_t n) { return (n + 63) / 64 * 64; };
  float* ws = static_cast<float*>(workspace(
      dev, stream, (r64(nq) + 2 * r64(nk) + r64(po_elems) + 2 * r64(ml_elems)) * sizeof(float)));
  if (ws == nullptr) return XATTN_ERR_NOMEM;
  float* q32 = ws;
  float* k32 = q32 + r64(nq);
  float* v32 = k32 + r64(nk);
  float* wpo = v32 + r64(nk);
  float* wpm = wpo + r64(po_elems);
  float* wpl = wpm + r64(ml_elems);
  const int sms = sm_count(dev);
  for (auto [src, dst, n] : {std::tuple<const __half*, float*, size_t>{Q, q32, nq},
                             {K, k32, nk}, {V, v32, nk}}) {
    if (n == 0) continue;
    // D % 64 == 0, so every tensor holds a whole number of 8-element groups
    const long long n8 = static_cast<long long>(n / 8);
    const unsigned blocks = static_cast<unsigned>(std::min<long long>((n8 + 255) / 256, sms * 8LL));
    simt::widen_half_kernel<<<blocks, 256, 0, stream>>>(reinterpret_cast<const uint4*>(src),
                                                        reinterpret_cast<float4*>(dst), n8);
  }
  if (cudaPeekAtLastError() != cudaSuccess) return XATTN_ERR_LAUNCH;
  if (S > 0) {
    rc = launch_fused(q32, k32, v32, nullptr, po, pm, pl, B, Nl, Ni, D, S, chunk16, 1, stream,
                      1.f, true);
    if (rc != XATTN_OK) return rc;
    return launch_combine(po, pm, pl, O, static_cast<long long>(rows), D, S, stream);
  }
  if (pair) return launch_fused_pair(q32, k32, v32, O, B, Nl, Ni, D, stream, 1.f, true);
  if (splits == 1)
    return launch_fused(q32, k32, v32, O, nullptr, nullptr, nullptr, B, Nl, Ni, D, 1, Ni, 0,
                        stream, 1.f, true);
  rc = launch_fused(q32, k32, v32, nullptr, wpo, wpm, wpl, B, Nl, Ni, D, splits, chunk, 1, stream,
                    1.f, true);
  if (rc != XATTN_OK) return rc;
  return launch_combine(wpo, wpm, wpl, O, static_cast<long long>(rows), D, splits, stream);
}

}  // namespace
}  // namespace xattn

using namespace xattn;

// ===================================================================== Part 1: upstream ABI
extern "C" void launch_naive_kernel(const float* Q, const float* K, const float* V, float* output,
                                    int batch_size, int N_latent, int N_input, int dim,
                                    cudaStream_t stream) {
  run_fp32(Q, K, V, output, batch_size, N_latent, N_input, dim, stream);
}

extern "C" void launch_parallel_kernel(const float* Q, const float* K, const float* V,
                                       float* output, int batch_size, int N_latent, int N_input,
                                       int dim, cudaStream_t stream) {
  run_fp32(Q, K, V, output, batch_size, N_latent, N_input, dim, stream);
}

extern "C" void launch_tiled_kernel(const float* Q, const float* K, const float* V, float* output,
                                    int batch_size, int N_latent, int N_input, int dim,
                                    cudaStream_t stream) {
  run_fp32(Q, K, V, output, batch_size, N_latent, N_input, dim, stream);
}

extern "C" void launch_optimized_kernel(const float* Q, const float* K, const float* V,
                                        float* output, int batch_size, int N_latent, int N_input,
                                        int dim, cudaStream_t stream) {
  run_fp32(Q, K, V, output, batch_size, N_latent, N_input, dim, stream);
}

extern "C" void launch_wmma_kernel(const __half* Q, const __half* K, const __half* V,
                                   float* output, int batch_size, int N_latent, int N_input,
                                   int dim, cudaStream_t stream) {
  if (bad_sizes(batch_size, N_latent, N_input, dim)) { set_error(XATTN_ERR_ARG); return; }
  if (batch_size == 0 || N_latent == 0) { set_error(XATTN_OK); return; }
  if (N_input == 0) { set_error(zero_output(output, batch_size, N_latent, dim, stream)); return; }
  if (Q == nullptr || K == nullptr || V == nullptr || output == nullptr) {
    set_error(XATTN_ERR_ARG);
    return;
  }
  // Q arrives pre-scaled by 1/sqrt(dim) (cuda_wrappers.py:635-640): score scale is 1.
  set_error(run_half(Q, K, V, output, nullptr, nullptr, nullptr, batch_size, N_latent, N_input,
                     dim, 0, stream));
}

extern "C" void launch_splitk_kernel(const float* Q, const float* K, const float* V, float* output,
                                     float* po, float* pm, float* pl, int batch_size, int N_latent,
                                     int N_input, int dim, int num_splits, cudaStream_t stream) {
  run_splitk(Q, K, V, output, po, pm, pl, batch_size, N_latent, N_input, dim, num_splits, stream);
}

extern "C" void launch_wmma_splitk_kernel(const __half* Q, const __half* K, const __half* V,
                                          float* output, float* po, float* pm, float* pl,
                                          int batch_size, int N_latent, int N_input, int dim,
                                          int num_splits, cudaStream_t stream) {
  if (bad_sizes(batch_size, N_latent, N_input, dim) || num_splits <= 0) {
    set_error(XATTN_ERR_ARG);
    return;
  }
  if (batch_size == 0 || N_latent == 0) { set_error(XATTN_OK); return; }
  if (output == nullptr || po == nullptr || pm == nullptr || pl == nullptr ||
      (N_input > 0 && (Q == nullptr || K == nullptr || V == nullptr))) {  // no keys: K, V unused
    set_error(XATTN_ERR_ARG);
    return;
  }
  if (N_input == 0) {
    int dev = 0;
    int rc = prepare_device(&dev);
    if (rc == XATTN_OK)
      rc = empty_partials(po, pm, pl, static_cast<long long>(batch_size) * N_latent * num_splits, dim, stream);
    set_error(rc != XATTN_OK ? rc : zero_output(output, batch_size, N_latent, dim, stream));
    return;
  }
  set_error(run_half(Q, K, V, output, po, pm, pl, batch_size, N_latent, N_input, dim, num_splits,
                     stream));
}

// ===================================================================== Part 2: new API
extern "C" int xattn_fp32(const float* Q, const float* K, const float* V, float* output,
                          int batch_size, int N_latent, int N_input, int dim,
                          cudaStream_t stream) {
  return run_fp32(Q, K, V, output, batch_size, N_latent, N_input, dim, stream);
}

extern "C" int xattn_fp32_partial(const float* Q, const float* K, const float* V, float* po,
                                  float* pm, float* pl, int batch_size, int N_latent,
                                  int N_input, int dim, cudaStream_t stream) {
  if (bad_sizes(batch_size, N_latent, N_input, dim)) return set_error(XATTN_ERR_ARG);
  if (batch_size == 0 || N_latent == 0) return set_error(XATTN_OK);
  if (po == nullptr || pm == nullptr || pl == nullptr) return set_error(XATTN_ERR_ARG);
  int dev = 0;
  int rc = prepare_device(&dev);
  if (rc != XATTN_OK) return set_error(rc);
  if (N_input == 0)  // a rank whose key slice is empty (N_input split over more ranks than keys)
    return set_error(empty_partials(po, pm, pl, static_cast<long long>(batch_size) * N_latent, dim, stream));
  const float scale_log2 = kLog2e / std::sqrt(static_cast<float>(dim));
  const int path = g_opt_path.load();
  if (path == 2 || !tc_fp32_supported(Q, K, V, po, dim))
    return set_error(launch_simt<float, float>(Q, K, V, nullptr, po, pm, pl, batch_size, 1, N_latent,
                                               N_input, dim, 1, std::max(1, N_input), 1,
                                               scale_log2, stream));
  // Key splits when the row blocks alone cannot fill the GPU, as for the plain entry; the
  // splits' partials are then merged into the one (m, l, O) triple asked for.
  return set_error(run_fused_auto(dev, Q, K, V, nullptr, po, pm, pl, batch_size, N_latent, N_input,
                                  dim, true, stream));
}

extern "C" int xattn_combine(const float* po, const float* pm, const float* pl, float* output,
                             long long rows, int dim, int num_splits, cudaStream_t stream) {
  if (rows < 0 || dim <= 0 || num_splits <= 0) return set_error(XATTN_ERR_ARG);
  return set_error(launch_combine(po, pm, pl, output, rows, dim, num_splits, stream));
}

extern "C" int xattn_lse_pack(const float* po, const float* pl, float* ol, long long rows, int dim,
                              cudaStream_t stream) {
  if (rows < 0 || dim <= 0) return set_error(XATTN_ERR_ARG);
  if (rows == 0) return set_error(XATTN_OK);
  simt::lse_pack_kernel<<<static_cast<unsigned>((rows + 3) / 4), 128, 0, stream>>>(po, pl, ol, rows,
                                                                                    dim);
  return set_error(cudaPeekAtLastError() == cudaSuccess ? XATTN_OK : XATTN_ERR_LAUNCH);
}

extern "C" int xattn_lse_rescale(float* ol, const float* pm, const float* m_glob, long long rows,
                                 int dim, cudaStream_t stream) {
  if (rows < 0 || dim <= 0) return set_error(XATTN_ERR_ARG);
  if (rows == 0) return set_error(XATTN_OK);
  simt::lse_rescale_kernel<<<static_cast<unsigned>((rows + 3) / 4), 128, 0, stream>>>(ol, pm, m_glob,
                                                                                       rows, dim);
  return set_error(cudaPeekAtLastError() == cudaSuccess ? XATTN_OK : XATTN_ERR_LAUNCH);
}

extern "C" int xattn_lse_finalize(const float* ol, float* output, long long rows, int dim,
                                  cudaStream_t stream) {
  if (rows < 0 || dim <= 0) return set_error(XATTN_ERR_ARG);
  if (rows == 0) return set_error(XATTN_OK);
  simt::lse_finalize_kernel<<<static_cast<unsigned>((rows + 3) / 4), 128, 0, stream>>>(ol, output,
                                                                                        rows, dim);
  return set_error(cudaPeekAtLastError() == cudaSuccess ? XATTN_OK : XATTN_ERR_LAUNCH);
}

// Multi-head bf16 tensor-core kernel (mha_bf16.cuh): heads side by side in rows of
// heads * head_dim elements.  Persistent: two CTAs per SM (the kernel's occupancy) loop
// over the B * heads * row-block items.  One instantiation per head dimension.
template <int kDh>
int launch_mha_bf16_dh(const __nv_bfloat16* Q, const __nv_bfloat16* K, const __nv_bfloat16* V,
                    __nv_bfloat16* out, int B, int Nl, int Ni, int heads, int dh, int sms,
                    cudaStream_t stream) {
  mha::Params p;
  const uint64_t ld = static_cast<uint64_t>(heads) * dh;
  const uint64_t dq[3] = {ld, (uint64_t)Nl, (uint64_t)B};
  const uint64_t sq[2] = {ld * 2, (uint64_t)Nl * ld * 2};
  const uint64_t dk[3] = {ld, (uint64_t)Ni, (uint64_t)B};
  const uint64_t sk[2] = {ld * 2, (uint64_t)Ni * ld * 2};
  using L = mha::Layout<kDh>;
  const CUtensorMapSwizzle swz = L::kRowB == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  const uint32_t bq[3] = {static_cast<uint32_t>(L::kBc), mha::kRows, 1};
  const uint32_t bk[3] = {static_cast<uint32_t>(L::kBc), mha::kKeys, 1};
  const uint32_t bo[3] = {32, 32, 1};  // output chunks of 32 rows x 32 columns
  if (!encode_tmap(&p.tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, Q, dq, sq, bq, swz) ||
      !encode_tmap(&p.tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, K, dk, sk, bk, swz) ||
      !encode_tmap(&p.tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, V, dk, sk, bk, swz) ||
      !encode_tmap(&p.to, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, out, dq, sq, bo,
                   CU_TENSOR_MAP_SWIZZLE_64B))
    return XATTN_ERR_ARG;
  p.heads = heads;
  p.n_latent = Nl;
  p.n_input = Ni;
  p.dh = dh;
  p.ld = static_cast<int>(ld);
  p.n_row_blocks = (Nl + mha::kRows - 1) / mha::kRows;
  p.scale_log2 = static_cast<float>(kLog2e / std::sqrt(static_cast<double>(dh)));
  const long long items = static_cast<long long>(B) * heads * p.n_row_blocks;
  if (items > 0x7fffffffLL) return XATTN_ERR_ARG;
  p.n_items = static_cast<int>(items);
  const long long ctas = std::min<long long>(items, 2LL * sms);
  mha::mha_bf16_kernel<kDh><<<static_cast<unsigned>(ctas), mha::kThreads, mha::kSmemBytes, stream>>>(p);
  return cudaPeekAtLastError() == cudaSuccess ? XATTN_OK : XATTN_ERR_LAUNCH;
}

int launch_mha_bf16(const __nv_bfloat16* Q, const __nv_bfloat16* K, const __nv_bfloat16* V,
                    __nv_bfloat16* out, int B, int Nl, int Ni, int heads, int dh, int sms,
                    cudaStream_t stream) {
  switch (dh) {
    case 32: return launch_mha_bf16_dh<32>(Q, K, V, out, B, Nl, Ni, heads, dh, sms, stream);
    case 64: return launch_mha_bf16_dh<64>(Q, K, V, out, B, Nl, Ni, heads, dh, sms, stream);
    case 96: return launch_mha_bf16_dh<96>(Q, K, V, out, B, Nl, Ni, heads, dh, sms, stream);
    case 128: return launch_mha_bf16_dh<128>(Q, K, V, out, B, Nl, Ni, heads, dh, sms, stream);
    default: return XATTN_ERR_ARG;  // callers check mha::supports_dh first
  }
}

extern "C" int xattn_bf16_mha(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                              const __nv_bfloat16* V, __nv_bfloat16* output, int batch_size,
                              int N_latent, int N_input, int heads, int head_dim,
                              cudaStream_t stream) {
  if (bad_sizes(batch_size, N_latent, N_input, head_dim) || heads <= 0)
    return set_error(XATTN_ERR_ARG);
  if (batch_size == 0 || N_latent == 0) return set_error(XATTN_OK);
  if (output == nullptr) return set_error(XATTN_ERR_ARG);
  if (N_input == 0) {  // softmax over no keys: zeros, as for the fp32 entries
    const size_t bytes = static_cast<size_t>(batch_size) * N_latent * heads * head_dim * sizeof(__nv_bfloat16);
    return set_error(cudaMemsetAsync(output, 0, bytes, stream) == cudaSuccess ? XATTN_OK : XATTN_ERR_LAUNCH);
  }
  int dev = 0;
  int rc = prepare_device(&dev);
  if (rc != XATTN_OK) return set_error(rc);
  if (g_opt_path.load() != 2 && mha::supports_dh(head_dim) && aligned16(Q) && aligned16(K) &&
      aligned16(V) && aligned16(output) && static_cast<long long>(heads) * head_dim <= 0x7fffffff)
    return set_error(launch_mha_bf16(Q, K, V, output, batch_size, N_latent, N_input, heads,
                                     head_dim, sm_count(dev), stream));
  const float scale_log2 = kLog2e / std::sqrt(static_cast<float>(head_dim));
  return set_error(launch_simt<__nv_bfloat16, __nv_bfloat16>(
      Q, K, V, output, nullptr, nullptr, nullptr, batch_size, heads, N_latent, N_input, head_dim, 1,
      N_input, 0, scale_log2, stream));
}

extern "C" int xattn_plan_fp32(int batch_size, int N_latent, int N_input, int dim,
                               int* num_splits) {
  int splits = 1, chunk = N_input;
  int launches = 0;
  if (batch_size > 0 && N_latent > 0 && N_input > 0 && dim > 0) {
    int dev = 0;
    if (prepare_device(&dev) != XATTN_OK) return -1;
    const bool tc = dim >= 64 && dim <= 2 * fused::kMaxDh && dim % 64 == 0 && g_opt_path.load() != 2;
    const bool pair = tc && g_opt_kernel.load() != 1 && pair4::supports_dh(dim / 2);  // as run_fused_auto
    if (pair)
      plan_pair_splits(dev, batch_size, N_latent, N_input, &splits, &chunk);
    else if (tc)
      plan_splits(dev, batch_size, N_latent, N_input, g_opt_path.load(), &splits, &chunk);
    launches = splits > 1 ? 2 : 1;
  } else if (batch_size > 0 && N_latent > 0 && N_input == 0) {
    launches = 1;  // the zero fill
  }
  if (num_splits != nullptr) *num_splits = splits;
  return launches;
}

extern "C" int xattn_last_error(void) { return t_last_error; }

extern "C" int xattn_status(int clear) {
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  int st = 0;
  if (cudaMemcpyFromSymbol(&st, g_status, sizeof(int)) != cudaSuccess) return -1;
  if (clear) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_status, &zero, sizeof(int));
  }
  return st;
}

extern "C" int xattn_set_option(int key, int value) {
  switch (key) {
    case 1: return g_opt_path.exchange(value);
    case 2: return g_opt_splits.exchange(value);
    case 3: return g_opt_wait_us.exchange(value > 0 ? value : 2000000);
    case 4: return g_opt_tf32_comp.exchange(value);
    case 5: return g_opt_kernel.exchange(value);
    case 6: return g_opt_accurate.exchange(value);
    default: return -1;
  }
}

namespace xattn {
namespace {
// Waits on an mbarrier that is initialised with one expected arrival that never comes.
__global__ void selftest_timeout_kernel() {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(smem_u32(&bar), 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (!mbar_wait(smem_u32(&bar), 0, kTimeoutInjected, &abort_flag)) {
      // give-up path taken: status already recorded by mbar_wait
    }
  }
  __syncthreads();
}
}  // namespace
}  // namespace xattn

extern "C" int xattn_selftest_timeout(int bound_us) {
  const int prev = g_opt_wait_us.exchange(bound_us > 0 ? bound_us : 1000);
  int dev = 0;
  int rc = prepare_device(&dev);
  int st = -1;
  if (rc == XATTN_OK) {
    selftest_timeout_kernel<<<1, 32>>>();
    st = xattn_status(1);
  }
  g_opt_wait_us.store(prev);
  prepare_device(&dev);
  return st;
}

extern "C" int xattn_version(void) { return kVersion; }

// ===================================================================== multi-GPU peer merge
extern "C" int xattn_ipc_alloc(size_t bytes, void** ptr, void* handle) {
  if (ptr == nullptr || handle == nullptr || bytes == 0) return set_error(XATTN_ERR_ARG);
  *ptr = nullptr;
  if (cudaMalloc(ptr, bytes) != cudaSuccess) {
    cudaGetLastError();
    return set_error(XATTN_ERR_NOMEM);
  }
  cudaIpcMemHandle_t h;
  if (cudaMemset(*ptr, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, *ptr) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(*ptr);
    *ptr = nullptr;
    return set_error(XATTN_ERR_LAUNCH);
  }
  static_assert(sizeof(h) == XATTN_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  return set_error(XATTN_OK);
}

extern "C" int xattn_ipc_open(const void* handle, void** ptr) {
  if (ptr == nullptr || handle == nullptr) return set_error(XATTN_ERR_ARG);
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  if (cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    cudaGetLastError();
    *ptr = nullptr;
    return set_error(XATTN_ERR_LAUNCH);
  }
  return set_error(XATTN_OK);
}

extern "C" int xattn_ipc_close(void* ptr) {
  return set_error(cudaIpcCloseMemHandle(ptr) == cudaSuccess ? XATTN_OK : XATTN_ERR_LAUNCH);
}

extern "C" int xattn_ipc_free(void* ptr) {
  return set_error(cudaFree(ptr) == cudaSuccess ? XATTN_OK : XATTN_ERR_LAUNCH);
}

extern "C" long long xattn_peer_layout(long long rows, int dim, long long* offsets) {
  if (rows < 0 || dim <= 0) return -1;
  const peer::Layout l = peer::layout(rows, dim);
  if (offsets != nullptr) {
    offsets[0] = l.pm;
    offsets[1] = l.pl;
    offsets[2] = l.po;
    offsets[3] = l.out;
  }
  return l.total * 4;
}

extern "C" int xattn_peer_merge(void* const* bases, int n_ranks, int rank, long long rows, int dim,
                                unsigned int epoch, cudaStream_t stream) {
  if (bases == nullptr || n_ranks < 1 || n_ranks > peer::kMaxRanks || rank >= n_ranks || rows < 0 ||
      dim <= 0 || rows > 0x7fffffffLL)
    return set_error(XATTN_ERR_ARG);
  int dev = 0;
  int rc = prepare_device(&dev);
  if (rc != XATTN_OK) return set_error(rc);
  peer::Params a = {};
  for (int p = 0; p < n_ranks; ++p) {
    if (bases[p] == nullptr || !aligned16(bases[p])) return set_error(XATTN_ERR_ARG);
    a.base[p] = static_cast<float*>(bases[p]);
  }
  a.rows = rows;
  a.dim = dim;
  a.n_ranks = n_ranks;
  a.rank = rank;
  a.epoch = epoch;
  a.lay = peer::layout(rows, dim);
  const long long mine = rank < 0 ? rows : rows * (rank + 1) / n_ranks - rows * rank / n_ranks;
  // a warp per (row, column segment), one wave of blocks (two per SM at the kernel's register
  // count); at least one block, so that every rank takes part in both barriers
  const long long nseg = (dim & 3) == 0 ? (dim + peer::kSegCols - 1) / peer::kSegCols : (dim + 31) / 32;
  const long long want = (mine * nseg + peer::kThreads / 32 - 1) / (peer::kThreads / 32);
  const unsigned blocks = static_cast<unsigned>(std::max<long long>(1, std::min<long long>(want, sm_count(dev) * 2LL)));
  // programmatic stream serialization: the launch and the blocks' start overlap the
  // partial's last kernel, which triggers its dependents early
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks);
  cfg.blockDim = dim3(peer::kThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return set_error(cudaLaunchKernelEx(&cfg, peer::merge_kernel, a) == cudaSuccess ? XATTN_OK : XATTN_ERR_LAUNCH);
}

#ifdef XATTN_TRACE
// Development builds only: copies the device timeline buffer to `host` (16*16*16 u64).
extern "C" int xattn_trace_fetch(unsigned long long* host) {
  return static_cast<int>(cudaMemcpyFromSymbol(host, g_trace, sizeof(g_trace)));
}
#endif

// ===================================================================== no-allocation split-K
// xattn_splitk_noalloc: the launch_splitk_kernel computation with its partials in a fixed
// scratch array that is part of the library image, for callers that may not allocate
// device memory during a call (see include/xattn.h).  The host never dereferences the
// array's symbol: it asks the runtime for the array's device address once per device.
namespace xattn {
namespace {

// The documented limit, B * N_latent * num_splits * (dim + 2) floats (32 MiB), plus room for
// the 256-byte alignment of the three sub-arrays (at most 3 * 63 floats), so that every
// request within the documented limit fits.
constexpr size_t kNoAllocLimitFloats = static_cast<size_t>(8) << 20;
constexpr size_t kNoAllocScratchFloats = kNoAllocLimitFloats + 192;
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

constexpr int kNoAllocDevices = 64;
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[kNoAllocDevices] = {};

// Device address of the scratch array on device `dev` (current), looked up on first use.
float* noalloc_scratch(int dev) {
  if (dev < 0 || dev >= kNoAllocDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || ptr == nullptr)
      return nullptr;
    g_noalloc_ptr[dev] = static_cast<float*>(ptr);
  }
  return g_noalloc_ptr[dev];
}

size_t round_up64(size_t n) { return (n + 63) / 64 * 64; }  // 256-byte sub-array alignment

}  // namespace
}  // namespace xattn

extern "C" int xattn_splitk_noalloc(const float* Q, const float* K, const float* V, float* output,
                                    int batch_size, int N_latent, int N_input, int dim,
                                    int num_splits, cudaStream_t stream) {
  if (bad_sizes(batch_size, N_latent, N_input, dim) || num_splits <= 0)
    return set_error(XATTN_ERR_ARG);
  if (batch_size == 0 || N_latent == 0) return set_error(XATTN_OK);
  if (output == nullptr) return set_error(XATTN_ERR_ARG);
  if (N_input == 0) return set_error(zero_output(output, batch_size, N_latent, dim, stream));
  if (Q == nullptr || K == nullptr || V == nullptr) return set_error(XATTN_ERR_ARG);
  const size_t rows = static_cast<size_t>(batch_size) * N_latent;  // >= 1, < 2^62
  // rows * num_splits * (dim + 2) <= capacity, tested by division so that no product can
  // wrap around (each factor is below 2^62 and 2^32)
  const size_t per_row = static_cast<size_t>(num_splits) * (static_cast<size_t>(dim) + 2);
  if (per_row > kNoAllocLimitFloats / rows) return set_error(XATTN_ERR_TOO_LARGE);
  const size_t po_elems = round_up64(rows * num_splits * dim);
  const size_t ml_elems = round_up64(rows * num_splits);
  if (po_elems + 2 * ml_elems > kNoAllocScratchFloats) return set_error(XATTN_ERR_TOO_LARGE);
  int dev = 0;
  int rc = prepare_device(&dev);
  if (rc != XATTN_OK) return set_error(rc);
  float* po = noalloc_scratch(dev);
  if (po == nullptr) return set_error(XATTN_ERR_LAUNCH);
  float* pm = po + po_elems;
  float* pl = pm + ml_elems;
  const int chunk = std::max(1, (N_input + num_splits - 1) / num_splits);  // kernel_splitk.cu:59
  const float scale_log2 = kLog2e / std::sqrt(static_cast<float>(dim));
  // the kernel choice of launch_splitk_kernel (run_splitk)
  if (g_opt_path.load() == 2 || !tc_fp32_supported(Q, K, V, output, dim))
    rc = launch_simt<float, float>(Q, K, V, nullptr, po, pm, pl, batch_size, 1, N_latent, N_input,
                                   dim, num_splits, chunk, 1, scale_log2, stream);
  else if (g_opt_kernel.load() != 1 && pair4::supports_dh(dim / 2))
    rc = launch_fused_pair<float>(Q, K, V, nullptr, po, pm, pl, batch_size, N_latent, N_input, dim,
                                  num_splits, chunk, 1, stream);
  else
    rc = launch_fused(Q, K, V, nullptr, po, pm, pl, batch_size, N_latent, N_input, dim,
                      num_splits, chunk, 1, stream);
  if (rc != XATTN_OK) return set_error(rc);
  return set_error(launch_combine(po, pm, pl, output, static_cast<long long>(rows), dim,
                                  num_splits, stream));
}
