"""PyTorch-facing API of the B200 cross-attention library (``kernels.so``).

Functions take CUDA tensors and launch on ``torch.cuda.current_stream()``:

* ``cross_attention(q, k, v)``          fp32 API, O = softmax(q k^T / sqrt(D)) v
  (the upstream ``compute_cross_attention`` contract, ``generate_batch_references.py:20-26``);
* ``cross_attention_splitk(q, k, v, num_splits)``  the upstream split-K entry with
  caller-visible (m, l, O) partials (``kernel_splitk.cu:42-251``);
* ``cross_attention_partial`` / ``combine``        partial triples and their merge;
* ``cross_attention_bf16_mha(q, k, v, heads)``     multi-head bf16 (no upstream counterpart);
* ``cross_attention_from_host(q, k, v)``  host-resident fp32 inputs and output, batch chunks
  pipelined through copy-in / compute / copy-out streams.

Multi-GPU (one process per GPU, ``torch.distributed``):

* ``shard_rows`` -- batch rows split contiguously over ranks; every rank runs the
  fused kernel on its own shard, no collective on the data path (weak scaling).
* ``cross_attention_input_split`` -- N_input split over ranks: each rank computes the
  partial (m, l, O) of its key slice into a peer-mapped exchange buffer (``PeerExchange``,
  CUDA IPC over NVLink) and ONE merge kernel per rank (``xattn_peer_merge``) exchanges and
  merges the partials over peer memory and leaves every row on every rank.
  ``merge_input_split`` is the same merge as NCCL collectives (all-reduce(MAX, m) ->
  rescale -> all-reduce(SUM, [O | l]) -> O / l), for process groups without peer memory
  (e.g. gloo) and as the comparison baseline.

Roofline formulas follow ``experiments/roofline.py:25-36`` upstream:
FLOPs = 4 B Nl Ni D, fused bytes = (2 Nl D + 2 Ni D) B elem.

The library must be built (``make`` in this directory); importing this module on a
machine without it raises, there is no CPU fallback.
"""

from __future__ import annotations

import ctypes
import math
import os
from typing import Callable, Optional, Sequence

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("XATTN_LIB", os.path.join(_HERE, "kernels.so"))

_lib = None

# Names every build of kernels.so exports (the contract of include/xattn.h).
EXPORTED = (
    "launch_naive_kernel", "launch_parallel_kernel", "launch_tiled_kernel",
    "launch_optimized_kernel", "launch_wmma_kernel", "launch_splitk_kernel",
    "launch_wmma_splitk_kernel", "xattn_fp32", "xattn_fp32_partial", "xattn_combine",
    "xattn_lse_pack", "xattn_lse_rescale", "xattn_lse_finalize", "xattn_bf16_mha",
    "xattn_last_error", "xattn_status", "xattn_set_option", "xattn_selftest_timeout",
    "xattn_version", "xattn_plan_fp32", "xattn_splitk_noalloc", "xattn_ipc_alloc", "xattn_ipc_open",
    "xattn_ipc_close", "xattn_ipc_free", "xattn_peer_layout", "xattn_peer_merge",
)

OPT_PATH, OPT_SPLITS, OPT_WAIT_US, OPT_TF32_COMP, OPT_KERNEL, OPT_ACCURATE = 1, 2, 3, 4, 5, 6


def lib():
    """Load kernels.so once and declare every exported signature."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} not found: build it with `make -C {_HERE}`")
    L = ctypes.CDLL(LIB_PATH)
    vp, i, ll = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong
    sig = {
        "launch_naive_kernel": ([vp] * 4 + [i] * 4 + [vp], None),
        "launch_parallel_kernel": ([vp] * 4 + [i] * 4 + [vp], None),
        "launch_tiled_kernel": ([vp] * 4 + [i] * 4 + [vp], None),
        "launch_optimized_kernel": ([vp] * 4 + [i] * 4 + [vp], None),
        "launch_wmma_kernel": ([vp] * 4 + [i] * 4 + [vp], None),
        "launch_splitk_kernel": ([vp] * 7 + [i] * 5 + [vp], None),
        "launch_wmma_splitk_kernel": ([vp] * 7 + [i] * 5 + [vp], None),
        "xattn_fp32": ([vp] * 4 + [i] * 4 + [vp], i),
        "xattn_fp32_partial": ([vp] * 6 + [i] * 4 + [vp], i),
        "xattn_combine": ([vp] * 4 + [ll, i, i, vp], i),
        "xattn_lse_pack": ([vp] * 3 + [ll, i, vp], i),
        "xattn_lse_rescale": ([vp] * 3 + [ll, i, vp], i),
        "xattn_lse_finalize": ([vp] * 2 + [ll, i, vp], i),
        "xattn_bf16_mha": ([vp] * 4 + [i] * 5 + [vp], i),
        "xattn_last_error": ([], i),
        "xattn_status": ([i], i),
        "xattn_set_option": ([i, i], i),
        "xattn_selftest_timeout": ([i], i),
        "xattn_version": ([], i),
        "xattn_plan_fp32": ([i, i, i, i, ctypes.POINTER(i)], i),
        "xattn_splitk_noalloc": ([vp] * 4 + [i] * 5 + [vp], i),
        "xattn_ipc_alloc": ([ctypes.c_size_t, ctypes.POINTER(vp), vp], i),
        "xattn_ipc_open": ([ctypes.c_char_p, ctypes.POINTER(vp)], i),
        "xattn_ipc_close": ([vp], i),
        "xattn_ipc_free": ([vp], i),
        "xattn_peer_layout": ([ll, i, ctypes.POINTER(ll)], ll),
        "xattn_peer_merge": ([vp, i, i, ll, i, ctypes.c_uint, vp], i),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res
    _lib = L
    return L


def set_option(key: int, value: int) -> int:
    return lib().xattn_set_option(key, value)


def plan_fp32(b: int, nl: int, ni: int, d: int):
    """(kernel launches per call, key splits) the fp32 entry will use for this shape."""
    n = ctypes.c_int(0)
    launches = lib().xattn_plan_fp32(b, nl, ni, d, ctypes.byref(n))
    return launches, n.value


def device_status(clear: bool = True) -> int:
    return lib().xattn_status(1 if clear else 0)


# ----------------------------------------------------------------------------- roofline
def flops(b: int, nl: int, ni: int, d: int) -> float:
    """Forward FLOPs of the two matmuls, 4 B Nl Ni D (upstream roofline.py:25-27)."""
    return 4.0 * b * nl * ni * d


def bytes_moved(b: int, nl: int, ni: int, d: int, elem: int = 4) -> float:
    """Fused HBM bytes, (2 Nl D + 2 Ni D) B elem (upstream roofline.py:30-36)."""
    return (2.0 * nl * d + 2.0 * ni * d) * b * elem


# ----------------------------------------------------------------------------- helpers
def _stream():
    import torch

    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _as3(x):
    return x.unsqueeze(0) if x.dim() == 2 else x


def _check_fp32(*ts):
    import torch

    for t in ts:
        if not t.is_cuda or t.dtype != torch.float32 or not t.is_contiguous():
            raise ValueError("expected contiguous float32 CUDA tensors")


def _raise(rc: int, what: str):
    if rc != 0:
        raise RuntimeError(f"{what} failed with xattn status {rc}")


# ----------------------------------------------------------------------------- single GPU
def cross_attention(q, k, v, out=None):
    """O = softmax(q k^T / sqrt(D)) v on the GPU (tcgen05 TF32 with fp32 accumulation)."""
    import torch

    squeeze = q.dim() == 2
    q, k, v = _as3(q), _as3(k), _as3(v)
    _check_fp32(q, k, v)
    b, nl, d = q.shape
    ni = k.shape[1]
    if out is None:
        out = torch.empty_like(q)
    _raise(lib().xattn_fp32(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), b, nl, ni,
                            d, _stream()), "xattn_fp32")
    return out[0] if squeeze else out


_COPY_STREAMS = {}
_HOST_BUFFERS = {}


def _copy_streams(dev):
    """(host->device, device->host) streams of a device, created once."""
    import torch

    if dev.index not in _COPY_STREAMS:
        _COPY_STREAMS[dev.index] = (torch.cuda.Stream(dev), torch.cuda.Stream(dev))
    return _COPY_STREAMS[dev.index]


HOST_CHUNKS = 2  # default number of batch chunks of cross_attention_from_host


def host_chunks(b: int, chunk: Optional[int] = None):
    """Batch ranges [(c0, c1), ...] of cross_attention_from_host: chunks of `chunk` batches
    (default ceil(b / HOST_CHUNKS))."""
    c = max(1, chunk or (b + HOST_CHUNKS - 1) // HOST_CHUNKS)
    return [(c0, min(b, c0 + c)) for c0 in range(0, b, c)]


def cross_attention_from_host(q, k, v, out=None, chunk: Optional[int] = None):
    """cross_attention for host-resident fp32 q [B,Nl,D], k, v [B,Ni,D]; returns a host tensor.

    The batch is processed in chunks through three CUDA streams: the host->device copy of
    chunk c+1 and the device->host copy of chunk c-1 run while chunk c computes, on the
    caller's current stream.  The two copy directions use separate copy engines, so a step
    costs about its host->device transfer instead of the sum of both transfers and the
    kernels.  Device buffers persist per device for the last shape used, two sets of each
    that alternate between calls: a call's copy-in waits only for the kernels of the call
    before the previous one, so copy-ins of consecutive calls follow each other without a
    gap, and a call's copy-out overlaps the next call's copy-in.  Every host->device copy
    has a fixed cost (~20 us measured on B200 over PCIe), so the default is a few large
    chunks.  Inputs should be in pinned memory (otherwise the copies are synchronous and
    nothing overlaps) and must not change until the caller's stream has passed the call;
    `out` (host, pinned if given) receives the result.  The call returns once the work is
    queued, with the caller's stream ordered after the last copy-out.
    chunk: batches per chunk (default: the batch in HOST_CHUNKS chunks).
    """
    import torch

    q, k, v = _as3(q), _as3(k), _as3(v)
    for t in (q, k, v):
        if t.device.type != "cpu" or t.dtype != torch.float32:
            raise ValueError("expected float32 host tensors")
    b = q.shape[0]
    dev = torch.device("cuda", torch.cuda.current_device())
    main = torch.cuda.current_stream(dev)
    s_in, s_out = _copy_streams(dev)
    if out is None:
        out = torch.empty(q.shape, dtype=torch.float32, pin_memory=True)
    key = (tuple(q.shape), tuple(k.shape))
    st = _HOST_BUFFERS.get(dev.index)
    if st is None or st["key"] != key:
        if st is not None:  # the old buffers are idle before they go back to the allocator
            main.wait_stream(s_in)
            main.wait_stream(s_out)

        def one_set():
            return {"q": torch.empty(q.shape, device=dev), "k": torch.empty(k.shape, device=dev),
                    "v": torch.empty(v.shape, device=dev), "o": torch.empty(q.shape, device=dev),
                    "computed": None}

        st = {"key": key, "sets": [one_set(), one_set()], "flip": 0}
        _HOST_BUFFERS[dev.index] = st
        s_in.wait_stream(main)   # buffers allocated on the caller's stream
        s_out.wait_stream(main)
    bs = st["sets"][st["flip"]]  # the other set may still be in use by the previous call
    st["flip"] ^= 1
    dq, dk, dv, do = bs["q"], bs["k"], bs["v"], bs["o"]
    if bs["computed"] is not None:
        s_in.wait_event(bs["computed"])  # the kernels of the call before the previous one
    done = None
    for c0, c1 in host_chunks(b, chunk):
        sl = slice(c0, c1)
        with torch.cuda.stream(s_in):
            dq[sl].copy_(q[sl], non_blocking=True)
            dk[sl].copy_(k[sl], non_blocking=True)
            dv[sl].copy_(v[sl], non_blocking=True)
            landed = torch.cuda.Event()
            landed.record(s_in)
        main.wait_event(landed)
        cross_attention(dq[sl], dk[sl], dv[sl], out=do[sl])
        done = torch.cuda.Event()
        done.record(main)
        s_out.wait_event(done)
        with torch.cuda.stream(s_out):
            out[sl].copy_(do[sl], non_blocking=True)
    bs["computed"] = done
    main.wait_stream(s_out)
    return out


def cross_attention_splitk(q, k, v, num_splits: int):
    """Upstream split-K entry: returns (out, po, pm, pl) with the upstream scratch layout."""
    import torch

    q, k, v = _as3(q), _as3(k), _as3(v)
    _check_fp32(q, k, v)
    b, nl, d = q.shape
    ni = k.shape[1]
    out = torch.empty_like(q)
    po = torch.empty(b, nl, num_splits, d, device=q.device, dtype=torch.float32)
    pm = torch.empty(b, nl, num_splits, device=q.device, dtype=torch.float32)
    pl = torch.empty_like(pm)
    L = lib()
    L.launch_splitk_kernel(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), po.data_ptr(),
                           pm.data_ptr(), pl.data_ptr(), b, nl, ni, d, num_splits, _stream())
    _raise(L.xattn_last_error(), "launch_splitk_kernel")
    return out, po, pm, pl


def cross_attention_partial(q, k, v):
    """Partial (m, l, O) of the keys in k/v: po [B,Nl,D], pm, pl [B,Nl] (natural-log units)."""
    import torch

    q, k, v = _as3(q), _as3(k), _as3(v)
    _check_fp32(q, k, v)
    b, nl, d = q.shape
    ni = k.shape[1]
    po = torch.empty_like(q)
    pm = torch.empty(b, nl, device=q.device, dtype=torch.float32)
    pl = torch.empty_like(pm)
    _raise(lib().xattn_fp32_partial(q.data_ptr(), k.data_ptr(), v.data_ptr(), po.data_ptr(),
                                    pm.data_ptr(), pl.data_ptr(), b, nl, ni, d, _stream()),
           "xattn_fp32_partial")
    return po, pm, pl


def combine(po, pm, pl):
    """Merge [..., S, D] partials into [..., D] (upstream kernel_splitk.cu:186-236)."""
    import torch

    s, d = po.shape[-2], po.shape[-1]
    rows = po.numel() // (s * d)
    out = torch.empty(po.shape[:-2] + (d,), device=po.device, dtype=torch.float32)
    _raise(lib().xattn_combine(po.data_ptr(), pm.data_ptr(), pl.data_ptr(), out.data_ptr(), rows, d,
                               s, _stream()), "xattn_combine")
    return out


def cross_attention_bf16_mha(q, k, v, heads: int, out=None):
    """Multi-head bf16 attention: [B,N,H*dh] inputs, heads contiguous, scale 1/sqrt(dh)."""
    import torch

    b, nl, dm = q.shape
    ni = k.shape[1]
    if dm % heads:
        raise ValueError("model width must be a multiple of heads")
    for t in (q, k, v):
        if not t.is_cuda or t.dtype != torch.bfloat16 or not t.is_contiguous():
            raise ValueError("expected contiguous bfloat16 CUDA tensors")
    if out is None:
        out = torch.empty_like(q)
    _raise(lib().xattn_bf16_mha(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), b, nl, ni,
                                heads, dm // heads, _stream()), "xattn_bf16_mha")
    return out


# ----------------------------------------------------------------------------- multi-GPU
def shard_rows(total: int, rank: int, world: int):
    """Contiguous [begin, end) slice of `total` items for `rank` of `world` (balanced)."""
    base, extra = divmod(total, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


class MergeOps:
    """The three device steps of the N_input merge; the default binds the CUDA kernels."""

    def pack(self, po, pl):
        import torch

        rows, d = pl.numel(), po.shape[-1]
        ol = torch.empty(rows, d + 1, device=po.device, dtype=torch.float32)
        _raise(lib().xattn_lse_pack(po.data_ptr(), pl.data_ptr(), ol.data_ptr(), rows, d, _stream()),
               "xattn_lse_pack")
        return ol

    def rescale(self, ol, pm, m_glob):
        _raise(lib().xattn_lse_rescale(ol.data_ptr(), pm.data_ptr(), m_glob.data_ptr(), ol.shape[0],
                                       ol.shape[1] - 1, _stream()), "xattn_lse_rescale")
        return ol

    def finalize(self, ol):
        import torch

        rows, d = ol.shape[0], ol.shape[1] - 1
        out = torch.empty(rows, d, device=ol.device, dtype=torch.float32)
        _raise(lib().xattn_lse_finalize(ol.data_ptr(), out.data_ptr(), rows, d, _stream()),
               "xattn_lse_finalize")
        return out


def merge_input_split(po, pm, pl, group=None, ops: Optional[MergeOps] = None):
    """Merge per-rank partials of disjoint key slices into the full attention output.

    Collective protocol (identical on every rank, same order):
      1. m_glob = all_reduce(MAX, pm)                     [rows] fp32
      2. ol = [po | pl] rescaled by exp(pm - m_glob)       local
      3. all_reduce(SUM, ol)                               [rows, D+1] fp32
      4. out = ol[:, :D] / ol[:, D]                         local
    Returns out with po's shape.
    """
    import torch.distributed as dist

    ops = ops or MergeOps()
    shape = po.shape
    pm_flat = pm.reshape(-1).contiguous()
    m_glob = pm_flat.clone()
    dist.all_reduce(m_glob, op=dist.ReduceOp.MAX, group=group)
    ol = ops.pack(po.reshape(-1, shape[-1]).contiguous(), pl.reshape(-1).contiguous())
    ol = ops.rescale(ol, pm_flat, m_glob)
    dist.all_reduce(ol, op=dist.ReduceOp.SUM, group=group)
    return ops.finalize(ol).reshape(shape)


class _DeviceArray:
    """Zero-copy torch view of device memory the library allocated."""

    def __init__(self, ptr: int, shape):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": "<f4", "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerExchange:
    """Exchange buffers of the N_input split over peer memory, one per rank of `group`.

    Every rank allocates its buffer (``xattn_ipc_alloc``), the 64-byte CUDA IPC handles go
    round with ``all_gather_object`` and every rank maps every other rank's buffer
    (``xattn_ipc_open``, NVLink peer access).  ``po`` / ``pm`` / ``pl`` are this rank's
    partial-output views (written by ``xattn_fp32_partial``), ``out`` the merged result
    [B, N_latent, D], valid until the next ``merge``.  One process per GPU of one node, at
    most eight ranks.  ``rows`` = B * N_latent.
    """

    def __init__(self, b: int, nl: int, d: int, group=None):
        import torch
        import torch.distributed as dist

        L = lib()
        self.group, self.shape = group, (b, nl, d)
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        if self.world > 8:
            raise ValueError("the peer merge takes at most eight ranks")
        self.rows, self.dim = b * nl, d
        offs = (ctypes.c_longlong * 4)()
        total = L.xattn_peer_layout(self.rows, d, offs)
        local, handle = ctypes.c_void_p(), ctypes.create_string_buffer(64)
        _raise(L.xattn_ipc_alloc(total, ctypes.byref(local), handle), "xattn_ipc_alloc")
        self.local = local.value
        handles = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=group)
        self.opened, ptrs = [], []
        for p, h in enumerate(handles):
            if p == self.rank:
                ptrs.append(self.local)
                continue
            peer = ctypes.c_void_p()
            _raise(L.xattn_ipc_open(h, ctypes.byref(peer)), "xattn_ipc_open")
            self.opened.append(peer.value)
            ptrs.append(peer.value)
        self.bases = (ctypes.c_void_p * self.world)(*ptrs)
        dev = torch.device("cuda", torch.cuda.current_device())

        def view(off, shape):
            return torch.as_tensor(_DeviceArray(self.local + int(off) * 4, shape), device=dev)

        self.pm, self.pl = view(offs[0], (b, nl)), view(offs[1], (b, nl))
        self.po, self.out = view(offs[2], (b, nl, d)), view(offs[3], (b, nl, d))
        self.epoch = 0
        torch.cuda.synchronize()  # the buffer is zeroed (flags at epoch 0) before any peer uses it
        dist.barrier(group=group)

    def partial(self, q, k_local, v_local):
        """This rank's (m, l, O) over its keys, into the exchange buffer."""
        q, k_local, v_local = _as3(q), _as3(k_local), _as3(v_local)
        _check_fp32(q, k_local, v_local)
        b, nl, d = q.shape
        if (b, nl, d) != self.shape:
            raise ValueError(f"exchange built for {self.shape}, got {(b, nl, d)}")
        _raise(lib().xattn_fp32_partial(q.data_ptr(), k_local.data_ptr(), v_local.data_ptr(),
                                        self.po.data_ptr(), self.pm.data_ptr(), self.pl.data_ptr(),
                                        b, nl, k_local.shape[1], d, _stream()), "xattn_fp32_partial")

    def merge(self):
        """One kernel: wait for every rank's partials, merge this rank's rows over peer memory
        into every rank's ``out``, wait for every rank.  Returns ``out``."""
        self.epoch += 1
        _raise(lib().xattn_peer_merge(self.bases, self.world, self.rank, self.rows, self.dim,
                                      self.epoch, _stream()), "xattn_peer_merge")
        return self.out

    def close(self):
        import torch
        import torch.distributed as dist

        torch.cuda.synchronize()
        dist.barrier(group=self.group)  # nobody reads or writes the buffers any more
        L = lib()
        for p in self.opened:
            L.xattn_ipc_close(p)
        dist.barrier(group=self.group)
        L.xattn_ipc_free(self.local)
        self.opened, self.local = [], None


_EXCHANGES = {}


def cross_attention_input_split(q, k_local, v_local, group=None, method: str = "peer"):
    """Attention over the union of every rank's key slice (N_input split across GPUs).

    method="peer": the partial into this rank's exchange buffer, then the one-kernel merge
    over peer memory (``PeerExchange``, cached per shape and group; the returned tensor is
    its ``out``, valid until the next call with that shape).  method="nccl": the merge as
    NCCL collectives (``merge_input_split``), a new tensor."""
    if method == "nccl":
        po, pm, pl = cross_attention_partial(q, k_local, v_local)
        return merge_input_split(po, pm, pl, group)
    q = _as3(q)
    key = (tuple(q.shape), group)
    ex = _EXCHANGES.get(key)
    if ex is None:
        ex = _EXCHANGES[key] = PeerExchange(*q.shape, group=group)
    ex.partial(q, k_local, v_local)
    return ex.merge()


def close_exchanges():
    """Unmaps and frees every cached PeerExchange (collective: every rank calls it)."""
    for ex in _EXCHANGES.values():
        ex.close()
    _EXCHANGES.clear()
