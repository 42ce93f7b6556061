"""ctypes binding of ``libdmoe_b200.so`` (the C ABI declared in ``include/dmoe_b200.h``) and
thin torch-tensor wrappers around it.

The shared library is the product's compute path.  There is no fallback: if the library is
missing or a call fails, these functions raise.  Tensors only supply device pointers,
sizes and the current CUDA stream; the kernels run inside the library.
"""

from __future__ import annotations

import ctypes
import os
import threading
from typing import Dict, Optional, Sequence, Tuple

import torch

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("DMOE_LIB", os.path.join(_PKG, "libdmoe_b200.so"))

F32, F16, BF16, E4M3 = 0, 1, 2, 3
TILES_AUTO, TILES_PAIR, TILES_SINGLE, TILES_PAIR_SPLIT = 0, 1, 2, 3
ACT_RELU, ACT_SILU = 0, 1
ROUTER_SOFTMAX, ROUTER_SIGMOID_GROUP = 0, 1

DEVERR_NAMES = {
    0x1: "grouped GEMM producer wait timed out",
    0x2: "grouped GEMM MMA wait timed out",
    0x4: "grouped GEMM epilogue wait timed out",
    0x8: "grouped GEMM teardown wait timed out",
    0x10: "completion flag wait timed out",
    0x20: "invalid segment table (clamped)",
    0x40: "expert-parallel flag wait timed out (a rank fell behind)",
    0x80: "expert-parallel receive buffer overflow (rows dropped)",
}

# Expert-parallel exchange (include/dmoe_b200.h, DMOE_EP_*).
EP_MAX_RANKS, EP_MAX_REPLICAS, EP_MAX_INSTANCES = 16, 4, 1024
EP_POLICY_ROTATE, EP_POLICY_SPLIT = 0, 1
EP_FLAG_COUNTS, EP_FLAG_DATA, EP_FLAG_RESULTS = 0, 1, 2


_DTYPE_CODE = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}

_vp = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_u64 = ctypes.c_uint64
_f32 = ctypes.c_float
_sz = ctypes.c_size_t


class EpWindow(ctypes.Structure):
    """``dmoe_ep_window``: every rank's flags, count matrix, receive rows, back map and return
    rows, as this process addresses them (its own memory, or CUDA-IPC mappings of the
    peers')."""
    _fields_ = [("world", ctypes.c_int32), ("rank", ctypes.c_int32),
                ("flags", _vp * EP_MAX_RANKS), ("counts", _vp * EP_MAX_RANKS),
                ("recv", _vp * EP_MAX_RANKS), ("back", _vp * EP_MAX_RANKS), ("rows", _vp * EP_MAX_RANKS)]

# name -> (restype, argtypes); mirrors include/dmoe_b200.h
SIGNATURES = {
    "dmoe_version": (ctypes.c_char_p, []),
    "dmoe_last_error": (ctypes.c_char_p, []),
    "dmoe_launch_count": (_u64, []),
    "dmoe_router": (ctypes.c_int, [_vp, _vp, ctypes.c_int, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                   ctypes.c_int, ctypes.c_int, ctypes.c_int, _f32, ctypes.c_int, ctypes.c_int, _vp,
                                   _vp, _vp, ctypes.c_int, _vp]),
    "dmoe_route_plan_workspace_size": (_sz, [ctypes.c_int, ctypes.c_int, ctypes.c_int]),
    "dmoe_route_plan": (ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp, _vp,
                                       _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "dmoe_route_plan_noalloc": (ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                               _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "dmoe_permute_rows": (ctypes.c_int, [_vp, _vp, _i64, _vp, _vp, _vp, _vp, ctypes.c_int, _vp]),
    "dmoe_grouped_mlp_workspace_size": (_sz, [ctypes.c_int, ctypes.c_int, ctypes.c_int]),
    "dmoe_grouped_gated_mlp_ex": (ctypes.c_int, [_vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                 ctypes.c_int, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                 ctypes.c_int, _vp, _vp, _sz, _vp, ctypes.c_int, _vp]),
    "dmoe_grouped_mlp_set_sm_reserve": (ctypes.c_int, [ctypes.c_int]),
    "dmoe_quantize_rows_e4m3": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int64, ctypes.c_int, _vp, ctypes.c_int64,
                                               _vp, ctypes.c_int64, _vp]),
    "dmoe_grouped_gated_mlp_fp8": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int,
                                                  ctypes.c_int, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                  ctypes.c_int, _vp, _vp, _sz, _vp, ctypes.c_int, _vp]),
    "dmoe_router_logits": (ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp, _vp,
                                          _vp]),
    "dmoe_grouped_gated_mlp": (ctypes.c_int, [_vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                              ctypes.c_int, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                              ctypes.c_int, _vp, _vp, _sz, _vp, _vp]),
    "dmoe_combine": (ctypes.c_int, [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                    ctypes.c_int, ctypes.c_int, _vp, _vp]),
    "dmoe_ipc_export": (ctypes.c_int, [_vp, _vp, ctypes.POINTER(_u64)]),
    "dmoe_ipc_open": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.POINTER(_vp)]),
    "dmoe_ipc_close": (ctypes.c_int, [_vp]),
    "dmoe_enable_peer_access": (ctypes.c_int, [ctypes.c_int, ctypes.c_int]),
    "dmoe_copy": (ctypes.c_int, [_vp, _vp, _sz, _vp]),
    "dmoe_flag_signal": (ctypes.c_int, [_vp, _u64, _vp]),
    "dmoe_flag_wait": (ctypes.c_int, [_vp, _u64, _u64, _vp, _vp]),
    "dmoe_ep_flags_bytes": (_sz, []),
    "dmoe_ep_counts_bytes": (_sz, [ctypes.c_int]),
    "dmoe_ep_plan": (ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp, _vp, _vp, _vp, _vp, _i64,
                                    _u64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "dmoe_ep_dispatch": (ctypes.c_int, [_vp, _vp, _i64, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp, _vp, _vp, _vp,
                                        _vp, _vp, _vp, _vp, _i64, _vp, _vp, _vp, _vp]),
    "dmoe_ep_expert_mlp": (ctypes.c_int, [_vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                          _vp, _vp, ctypes.c_int, _i64, ctypes.c_int, _vp, _sz, _vp, ctypes.c_int,
                                          _vp]),
    "dmoe_ep_expert_mlp_fp8": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                              _vp, _vp, ctypes.c_int, _i64, ctypes.c_int, _vp, _sz, _vp, ctypes.c_int,
                                              _vp]),
    "dmoe_ep_wait": (ctypes.c_int, [_vp, ctypes.c_int, _u64, _vp, _vp]),
    "dmoe_ep_signal": (ctypes.c_int, [_vp, ctypes.c_int, _vp]),
    "dmoe_ep_combine": (ctypes.c_int, [_vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                       ctypes.c_int, ctypes.c_int, _vp, _vp]),
    "dmoe_event_create": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.POINTER(_vp)]),
    "dmoe_event_destroy": (ctypes.c_int, [_vp]),
    "dmoe_event_record": (ctypes.c_int, [_vp, _vp]),
    "dmoe_event_query": (ctypes.c_int, [_vp]),
    "dmoe_stream_wait_event": (ctypes.c_int, [_vp, _vp]),
    "dmoe_ipc_event_export": (ctypes.c_int, [_vp, _vp]),
    "dmoe_ipc_event_open": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.POINTER(_vp)]),
}

_lib: Optional[ctypes.CDLL] = None
_lib_setup: Optional[ctypes.CDLL] = None
_lib_lock = threading.Lock()


class DMoEError(RuntimeError):
    pass


def lib() -> ctypes.CDLL:
    """Load the library once; raise if it is absent (the product has no CPU fallback)."""
    global _lib
    if _lib is None:
        with _lib_lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise DMoEError(f"{LIB_PATH} is missing: build it with `python -m distributedmoe_b200._build`")
                # Launches, copies and event operations only enqueue work, so these calls
                # keep the GIL (PyDLL): releasing and re-taking it around each call hands the
                # interpreter to another thread (the host's and the expert blocks' event loops
                # share a process) at every launch.
                _lib = _load(ctypes.PyDLL)
    return _lib


def lib_setup() -> ctypes.CDLL:
    """The same library with the GIL released during calls, for set-up calls that can take
    milliseconds (IPC mappings, events of another GPU, which may create its context)."""
    global _lib_setup
    if _lib_setup is None:
        lib()
        with _lib_lock:
            if _lib_setup is None:
                _lib_setup = _load(ctypes.CDLL)
    return _lib_setup


def _load(kind) -> ctypes.CDLL:
    handle = kind(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(handle, name)
        fn.restype = res
        fn.argtypes = args
    return handle


def _check(rc: int, what: str) -> None:
    if rc != 0:
        msg = lib().dmoe_last_error().decode(errors="replace")
        raise DMoEError(f"{what} failed (status {rc}): {msg}")


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dt]
    except KeyError:
        raise DMoEError(f"unsupported dtype {dt}") from None


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*ts: Optional[torch.Tensor]) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise DMoEError("dmoe kernels take CUDA tensors only (no CPU fallback)")
        if not t.is_contiguous():
            raise DMoEError("dmoe kernels take contiguous tensors")
        dev = t.device if dev is None else dev
    return dev


# ----------------------------------------------------------------------------- scratch
class _Scratch:
    """Per-(device, stream) growable scratch buffers and a per-device status word."""

    def __init__(self):
        self._bufs: Dict[Tuple[int, int, str], torch.Tensor] = {}
        self._status: Dict[int, torch.Tensor] = {}
        self._lock = threading.Lock()

    def get(self, device: torch.device, name: str, nbytes: int) -> torch.Tensor:
        key = (device.index, _stream(device), name)
        with self._lock:
            buf = self._bufs.get(key)
            if buf is None or buf.numel() < nbytes:
                buf = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)
                self._bufs[key] = buf
            return buf

    def status(self, device: torch.device) -> torch.Tensor:
        with self._lock:
            st = self._status.get(device.index)
            if st is None:
                st = torch.zeros(1, dtype=torch.int32, device=device)
                self._status[device.index] = st
            return st


scratch = _Scratch()


# ----------------------------------------------------------------------------- timing
_timing: Optional[Dict[str, list]] = None
_timing_lock = threading.Lock()


def enable_kernel_timing(on: bool = True) -> None:
    """Record CUDA events around every library op (per op name) until disabled."""
    global _timing
    with _timing_lock:
        _timing = {} if on else None


def kernel_times_ms() -> Dict[str, list]:
    """Durations (ms) of the ops recorded since timing was enabled; synchronises."""
    return {name: [ms for ms, _ in recs] for name, recs in kernel_records().items()}


def kernel_records() -> Dict[str, list]:
    """(duration ms, work) per recorded op; work is the op's algorithmic FLOPs where the
    wrapper knows them (the grouped MLP with a host segment table), else None."""
    with _timing_lock:
        snap = dict(_timing or {})
    out = {}
    for name, recs in snap.items():
        out[name] = []
        for a, b, work in recs:
            b.synchronize()
            out[name].append((a.elapsed_time(b), work))
    return out


class _Timed:
    __slots__ = ("name", "stream", "ev", "work")

    def __init__(self, name: str, stream: int, device: torch.device, work: Optional[float] = None):
        self.name = name
        self.ev = None
        self.work = work
        if _timing is not None and not torch.cuda.is_current_stream_capturing():
            # The current stream as torch knows it (the legacy default stream included);
            # another handle is wrapped.
            cur = torch.cuda.current_stream(device)
            self.stream = cur if cur.cuda_stream == stream else torch.cuda.ExternalStream(stream, device=device)
            self.ev = torch.cuda.Event(enable_timing=True)
            self.ev.record(self.stream)

    def done(self) -> None:
        if self.ev is not None:
            end = torch.cuda.Event(enable_timing=True)
            end.record(self.stream)
            with _timing_lock:
                if _timing is not None:
                    _timing.setdefault(self.name, []).append((self.ev, end, self.work))


def check_device_status(device: torch.device, reset: bool = True) -> None:
    """Raise if a kernel on `device` reported a timed-out wait or a bad segment table.
    Synchronises with the device status word (a 4-byte read)."""
    st = scratch.status(device)
    v = int(st.item())
    if v:
        if reset:
            st.zero_()
        names = [n for bit, n in DEVERR_NAMES.items() if v & bit]
        raise DMoEError(f"device reported error 0x{v:x}: {', '.join(names)}")


# ----------------------------------------------------------------------------- ops
# From this many experts on, bf16/f16 router logits are a tensor-core GEMM (dmoe_router_logits).
TC_LOGITS_MIN_EXPERTS = 32


def router(x: Optional[torch.Tensor], w_r: Optional[torch.Tensor], top_k: int, *, num_experts: Optional[int] = None,
           mode: int = ROUTER_SOFTMAX, renormalize: bool = False, scale: float = 1.0,
           logit_bias: Optional[torch.Tensor] = None, score_bias: Optional[torch.Tensor] = None, n_group: int = 1,
           topk_group: int = 1, logits_in: Optional[torch.Tensor] = None, want_logits: bool = False,
           w_dtype: Optional[torch.dtype] = None, out: Optional[Tuple[torch.Tensor, torch.Tensor]] = None):
    """Router kernel: returns (selected [T,k] int64, weights [T,k], logits [T,E] fp32 or None)."""
    if logits_in is not None:
        dev = _require_cuda(logits_in)
        T, E = logits_in.shape
        x_dtype = torch.float32
        d = 0
    else:
        dev = _require_cuda(x, w_r)
        T, d = x.shape
        E = w_r.shape[0]
        x_dtype = x.dtype
        if w_r.dtype != x.dtype or w_r.shape[1] != d:
            raise DMoEError("router weight must be [E, d] in the dtype of x")
    if num_experts is not None and num_experts != E:
        raise DMoEError("num_experts mismatch")
    w_dtype = w_dtype or (x_dtype if logits_in is None else torch.float32)
    if out is not None:
        idx, w = out
    else:
        idx = torch.empty(T, top_k, dtype=torch.int64, device=dev)
        w = torch.empty(T, top_k, dtype=w_dtype, device=dev)
    for b in (logit_bias, score_bias):
        if b is not None and (b.dtype != torch.float32 or b.numel() != E):
            raise DMoEError("router biases must be fp32 [E]")
    if logits_in is None and x_dtype in (torch.bfloat16, torch.float16) and E >= TC_LOGITS_MIN_EXPERTS \
            and E % 8 == 0 and d % 8 == 0 and E <= 256:
        # Many experts: the logits GEMM on the tensor cores, then selection from those logits.
        logits_in = torch.empty(T, E, dtype=torch.float32, device=dev)
        tm = _Timed("router_logits", _stream(dev), dev, 2.0 * T * d * E)
        _check(lib().dmoe_router_logits(x.data_ptr(), w_r.data_ptr(), dtype_code(x_dtype), T, d, E, logits_in.data_ptr(),
                                        scratch.status(dev).data_ptr(), _stream(dev)), "dmoe_router_logits")
        tm.done()
        if logit_bias is not None:
            logits_in.add_(logit_bias)
        logit_bias = None
        x = w_r = None
        x_dtype, d = torch.float32, 0
        logits = logits_in if want_logits else None
    else:
        logits = torch.empty(T, E, dtype=torch.float32, device=dev) if (want_logits and logits_in is None) else None
    tm = _Timed("router", _stream(dev), dev)
    rc = lib().dmoe_router(_ptr(x) if logits_in is None else None, _ptr(w_r) if logits_in is None else None,
                           dtype_code(x_dtype), _ptr(logit_bias), _ptr(score_bias), _ptr(logits_in), T, d, E, top_k,
                           mode, int(renormalize), float(scale), n_group, topk_group, _ptr(logits), idx.data_ptr(),
                           w.data_ptr(), dtype_code(w.dtype), _stream(dev))
    _check(rc, "dmoe_router")
    tm.done()
    return idx, w, logits


def route_plan(idx: torch.Tensor, w: Optional[torch.Tensor], num_experts: int, *, want_slot: bool = True,
               want_inverse: bool = True, want_weight: bool = True) -> Dict[str, torch.Tensor]:
    """Routing-plan kernels: counts, offsets, perm_token (+ perm_slot, inverse, perm_weight)."""
    dev = _require_cuda(idx, w)
    if idx.dtype != torch.int64:
        raise DMoEError("selected experts must be int64")
    T, k = idx.shape
    n = T * k
    E = num_experts
    res = {
        "counts": torch.empty(E, dtype=torch.int32, device=dev),
        "offsets": torch.empty(E + 1, dtype=torch.int32, device=dev),
        "perm_token": torch.empty(n, dtype=torch.int32, device=dev),
    }
    if want_slot:
        res["perm_slot"] = torch.empty(n, dtype=torch.int32, device=dev)
    if want_inverse:
        res["inverse"] = torch.empty(n, dtype=torch.int32, device=dev)
    if want_weight and w is not None:
        res["perm_weight"] = torch.empty(n, dtype=w.dtype, device=dev)
    ws_bytes = lib().dmoe_route_plan_workspace_size(T, k, E)
    ws = scratch.get(dev, "plan", ws_bytes)
    tm = _Timed("route_plan", _stream(dev), dev)
    rc = lib().dmoe_route_plan(idx.data_ptr(), _ptr(w), dtype_code(w.dtype) if w is not None else BF16, T, k, E,
                               res["counts"].data_ptr(), res["offsets"].data_ptr(), res["perm_token"].data_ptr(),
                               _ptr(res.get("perm_slot")), _ptr(res.get("inverse")), _ptr(res.get("perm_weight")),
                               ws.data_ptr(), ws.numel(), _stream(dev))
    _check(rc, "dmoe_route_plan")
    tm.done()
    return res


def _i32_array(vals: Sequence[int]):
    arr = (ctypes.c_int32 * max(len(vals), 1))(*[int(v) for v in vals])
    return arr


def permute_rows(src: torch.Tensor, dst: torch.Tensor, seg_src: Sequence[int], seg_dst: Sequence[int],
                 seg_len: Sequence[int], row_map: Optional[torch.Tensor] = None, dst_ptr: Optional[int] = None,
                 stream: Optional[int] = None) -> None:
    """dst[seg_dst[i] + r] = src[row_map[seg_src[i] + r] if row_map else seg_src[i] + r].
    ``dst_ptr`` overrides dst's pointer (a peer GPU buffer), keeping dst for shape/dtype."""
    dev = _require_cuda(src, row_map)
    row_bytes = src.shape[-1] * src.element_size()
    if dst.shape[-1] * dst.element_size() != row_bytes:
        raise DMoEError("src and dst rows differ in size")
    n = len(seg_len)
    st = stream if stream is not None else _stream(dev)
    tm = _Timed("permute_rows", st, dev)
    rc = lib().dmoe_permute_rows(src.data_ptr(), dst_ptr if dst_ptr is not None else dst.data_ptr(), row_bytes,
                                 _ptr(row_map), _i32_array(seg_src), _i32_array(seg_dst), _i32_array(seg_len), n,
                                 st)
    _check(rc, "dmoe_permute_rows")
    tm.done()


def grouped_gated_mlp(X: torch.Tensor, w_gate: torch.Tensor, w_up: torch.Tensor, w_down: torch.Tensor,
                      seg_expert, seg_end, act: int, Y: torch.Tensor, m_rows: Optional[int] = None,
                      op_name: str = "grouped_gated_mlp", tile_policy: int = TILES_AUTO) -> None:
    """Grouped expert MLP over row segments.  seg_expert/seg_end: Python int sequences (host
    table) or int32 CUDA tensors (device table)."""
    _require_cuda(X, Y)
    if X.shape[1] != w_gate.shape[2] or Y.shape[1] != w_gate.shape[2]:
        raise DMoEError("X and Y must be [rows, d]")
    if not (X.dtype == w_gate.dtype == Y.dtype):
        raise DMoEError("grouped MLP operands must share one dtype")
    m = X.shape[0] if m_rows is None else m_rows
    if m > X.shape[0] or m > Y.shape[0]:
        raise DMoEError("m_rows exceeds the rows of X or Y")
    grouped_gated_mlp_ptrs(X.data_ptr(), Y.data_ptr(), m, w_gate, w_up, w_down, seg_expert, seg_end, act, op_name,
                           tile_policy)


def grouped_gated_mlp_ptrs(x_ptr: int, y_ptr: int, m_rows: int, w_gate: torch.Tensor, w_up: torch.Tensor,
                           w_down: torch.Tensor, seg_expert, seg_end, act: int,
                           op_name: str = "grouped_gated_mlp", tile_policy: int = TILES_AUTO) -> None:
    """Same as :func:`grouped_gated_mlp` on raw device pointers (rows of d elements of the
    weights' dtype), e.g. a transfer-engine buffer of another block on this GPU."""
    dev = _require_cuda(w_gate, w_up, w_down)
    E, I, d = w_gate.shape
    if w_up.shape != (E, I, d) or w_down.shape != (E, d, I):
        raise DMoEError("expert stacks must be gate/up [E, I, d] and down [E, d, I]")
    if not (w_gate.dtype == w_up.dtype == w_down.dtype):
        raise DMoEError("grouped MLP operands must share one dtype")
    dt = dtype_code(w_gate.dtype)
    ws = scratch.get(dev, "mlp", lib().dmoe_grouped_mlp_workspace_size(m_rows, I, dt))
    work = None
    if isinstance(seg_expert, torch.Tensor):
        n_seg = seg_expert.numel()
        se, sn, on_dev = seg_expert.data_ptr(), seg_end.data_ptr(), 1
        keep = None
    else:
        n_seg = len(seg_expert)
        a1, a2 = _i32_array(seg_expert), _i32_array(seg_end)
        se, sn, on_dev = ctypes.addressof(a1), ctypes.addressof(a2), 0
        keep = (a1, a2)
        if _timing is not None:  # rows of real (expert >= 0) segments x 6 d I
            rows, start = 0, 0
            for e, end in zip(seg_expert, seg_end):
                if e >= 0:
                    rows += end - start
                start = end
            work = 6.0 * rows * d * I
    tm = _Timed(op_name, _stream(dev), dev, work)
    rc = lib().dmoe_grouped_gated_mlp_ex(x_ptr, w_gate.data_ptr(), w_up.data_ptr(), w_down.data_ptr(), E, d, I, dt,
                                         se, sn, n_seg, on_dev, m_rows, act, y_ptr, ws.data_ptr(), ws.numel(),
                                         scratch.status(dev).data_ptr(), int(tile_policy), _stream(dev))
    del keep
    _check(rc, "dmoe_grouped_gated_mlp")
    tm.done()


def quantize_rows_e4m3(x: torch.Tensor, q: Optional[torch.Tensor] = None,
                       scale: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Row-wise e4m3 quantisation of x [..., cols]: returns q (float8_e4m3fn, x's shape) and
    scale (fp32, one per row), x ~= q * scale[row]."""
    dev = _require_cuda(x)
    if not x.is_contiguous():
        raise DMoEError("x must be contiguous")
    cols = x.shape[-1]
    rows = x.numel() // cols if cols else 0
    if q is None:
        q = torch.empty(x.shape, dtype=torch.float8_e4m3fn, device=x.device)
    if scale is None:
        scale = torch.empty(x.shape[:-1], dtype=torch.float32, device=x.device)
    if q.dtype != torch.float8_e4m3fn or q.shape != x.shape or scale.numel() != rows or scale.dtype != torch.float32:
        raise DMoEError("q must be float8_e4m3fn of x's shape and scale fp32 with one value per row")
    tm = _Timed("quantize_rows_e4m3", _stream(dev), dev)
    rc = lib().dmoe_quantize_rows_e4m3(x.data_ptr(), dtype_code(x.dtype), rows, cols, q.data_ptr(), cols,
                                       scale.data_ptr(), 1, _stream(dev))
    _check(rc, "dmoe_quantize_rows_e4m3")
    tm.done()
    return q, scale


def fp8_record_bytes(d: int) -> int:
    """Bytes of one 8-bit receive record: d e4m3 codes, the row's fp32 scale, padding to 16."""
    return d + 16


def quantize_records(x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """x [T, d] -> uint8 records [T, d + 16]: row t's e4m3 codes, then its fp32 scale."""
    dev = _require_cuda(x)
    T, d = x.shape
    if d % 16:
        raise DMoEError(f"8-bit records need d % 16 == 0 (d={d})")
    if out is None:
        out = torch.empty(T, d + 16, dtype=torch.uint8, device=x.device)
    if out.dtype != torch.uint8 or out.shape[0] < T or out.shape[1] != d + 16 or not out.is_contiguous():
        raise DMoEError("records must be a contiguous uint8 [T, d + 16] tensor")
    if T == 0:
        return out
    tm = _Timed("quantize_rows_e4m3", _stream(dev), dev)
    rc = lib().dmoe_quantize_rows_e4m3(x.data_ptr(), dtype_code(x.dtype), T, d, out.data_ptr(), d + 16,
                                       out.data_ptr() + d, (d + 16) // 4, _stream(dev))
    _check(rc, "dmoe_quantize_rows_e4m3")
    tm.done()
    return out


class Fp8Experts:
    """An expert stack with e4m3 gate/up weights (one fp32 scale per output channel) and a
    bf16 down projection, quantised once from 16-bit stacks."""

    def __init__(self, w_gate: torch.Tensor, w_up: torch.Tensor, w_down: torch.Tensor) -> None:
        E, I, d = w_gate.shape
        if d % 16:
            raise DMoEError(f"8-bit experts need d % 16 == 0 (d={d})")
        if w_up.shape != (E, I, d) or w_down.shape != (E, d, I):
            raise DMoEError("expert stacks must be gate/up [E, I, d] and down [E, d, I]")
        self.wg_q, self.wg_scale = quantize_rows_e4m3(w_gate.contiguous())
        self.wu_q, self.wu_scale = quantize_rows_e4m3(w_up.contiguous())
        self.w_down = w_down.to(torch.bfloat16).contiguous()

    @property
    def shape(self):
        return self.wg_q.shape


def grouped_gated_mlp_fp8(Xq: torch.Tensor, x_scale: torch.Tensor, experts: Fp8Experts, seg_expert, seg_end,
                          act: int, Y: torch.Tensor, m_rows: Optional[int] = None,
                          tile_policy: int = TILES_AUTO) -> None:
    """Grouped expert MLP with an e4m3 gate/up GEMM (row and column scales applied in the
    activation epilogue) and a bf16 down GEMM.  Xq [rows, d] e4m3 with x_scale [rows];
    Y [rows, d] bf16.  seg_expert/seg_end as :func:`grouped_gated_mlp`."""
    dev = _require_cuda(Xq, x_scale, experts.wg_q, experts.w_down, Y)
    E, I, d = experts.wg_q.shape
    if Xq.dtype != torch.float8_e4m3fn or x_scale.dtype != torch.float32:
        raise DMoEError("Xq must be float8_e4m3fn with fp32 row scales")
    if Y.dtype != torch.bfloat16:
        raise DMoEError("Y must be bf16")
    if Xq.shape[1] != d or Y.shape[1] != d:
        raise DMoEError("Xq and Y must be [rows, d]")
    m = Xq.shape[0] if m_rows is None else m_rows
    if m > Xq.shape[0] or m > Y.shape[0] or m > x_scale.numel():
        raise DMoEError("m_rows exceeds the rows of Xq, x_scale or Y")
    ws = scratch.get(dev, "mlp", lib().dmoe_grouped_mlp_workspace_size(m, I, BF16))
    if isinstance(seg_expert, torch.Tensor):
        n_seg = seg_expert.numel()
        se, sn, on_dev, keep = seg_expert.data_ptr(), seg_end.data_ptr(), 1, None
    else:
        n_seg = len(seg_expert)
        a1, a2 = _i32_array(seg_expert), _i32_array(seg_end)
        se, sn, on_dev, keep = ctypes.addressof(a1), ctypes.addressof(a2), 0, (a1, a2)
    tm = _Timed("grouped_gated_mlp_fp8", _stream(dev), dev)
    rc = lib().dmoe_grouped_gated_mlp_fp8(Xq.data_ptr(), x_scale.data_ptr(), experts.wg_q.data_ptr(),
                                          experts.wg_scale.data_ptr(), experts.wu_q.data_ptr(),
                                          experts.wu_scale.data_ptr(), experts.w_down.data_ptr(), E, d, I, se, sn,
                                          n_seg, on_dev, m, act, Y.data_ptr(), ws.data_ptr(), ws.numel(),
                                          scratch.status(dev).data_ptr(), int(tile_policy), _stream(dev))
    del keep
    _check(rc, "dmoe_grouped_gated_mlp_fp8")
    tm.done()


def set_gemm_sm_reserve(sms: int) -> None:
    """SMs that later grouped-MLP launches of this process leave free for other streams."""
    _check(lib().dmoe_grouped_mlp_set_sm_reserve(int(sms)), "dmoe_grouped_mlp_set_sm_reserve")


def combine(rows: torch.Tensor, inverse: torch.Tensor, w: torch.Tensor, out: torch.Tensor,
            accumulate: bool = False) -> None:
    """out[t] = (out[t] if accumulate) + sum_s w[t,s] * rows[inverse[t*k+s]] (fp32 accumulate)."""
    dev = _require_cuda(rows, inverse, w, out)
    T, k = w.shape
    d = out.shape[-1]
    if rows.dtype != out.dtype:
        raise DMoEError("rows and out must share a dtype")
    tm = _Timed("combine", _stream(dev), dev)
    rc = lib().dmoe_combine(rows.data_ptr(), inverse.data_ptr(), w.data_ptr(), dtype_code(w.dtype), T, k, d,
                            dtype_code(out.dtype), int(accumulate), out.data_ptr(), _stream(dev))
    _check(rc, "dmoe_combine")
    tm.done()


# ----------------------------------------------------------------------------- transfer
def ipc_export(ptr: int) -> Tuple[bytes, int]:
    """(64-byte handle of the allocation holding ptr, byte offset of ptr inside it)."""
    buf = (ctypes.c_uint8 * 64)()
    off = _u64()
    _check(lib_setup().dmoe_ipc_export(ptr, buf, ctypes.byref(off)), "dmoe_ipc_export")
    return bytes(buf), int(off.value)


def ipc_open(handle: bytes, device: int) -> int:
    if len(handle) != 64:
        raise DMoEError("IPC handle must be 64 bytes")
    buf = (ctypes.c_uint8 * 64).from_buffer_copy(handle)
    out = _vp()
    _check(lib_setup().dmoe_ipc_open(buf, device, ctypes.byref(out)), "dmoe_ipc_open")
    return int(out.value)


def ipc_close(ptr: int) -> None:
    _check(lib_setup().dmoe_ipc_close(ptr), "dmoe_ipc_close")


def enable_peer_access(device: int, peer: int) -> None:
    _check(lib_setup().dmoe_enable_peer_access(device, peer), "dmoe_enable_peer_access")


DMOE_NOT_READY = 4


def event_create(device: int, interprocess: bool = False) -> int:
    """A raw CUDA event (timing disabled) of `device`; returns its handle as an int."""
    out = _vp()
    _check(lib_setup().dmoe_event_create(device, int(interprocess), ctypes.byref(out)), "dmoe_event_create")
    return int(out.value)


def event_destroy(event: int) -> None:
    _check(lib_setup().dmoe_event_destroy(event), "dmoe_event_destroy")


def event_record(event: int, stream: int) -> None:
    _check(lib().dmoe_event_record(event, stream), "dmoe_event_record")


def event_query(event: int) -> bool:
    """True when the work before the event's last record has finished."""
    rc = lib().dmoe_event_query(event)
    if rc == DMOE_NOT_READY:
        return False
    _check(rc, "dmoe_event_query")
    return True


def stream_wait_event(stream: int, event: int) -> None:
    _check(lib().dmoe_stream_wait_event(stream, event), "dmoe_stream_wait_event")


def ipc_event_export(event: int) -> bytes:
    buf = (ctypes.c_uint8 * 64)()
    _check(lib_setup().dmoe_ipc_event_export(event, buf), "dmoe_ipc_event_export")
    return bytes(buf)


def ipc_event_open(handle: bytes, device: int) -> int:
    """Open another process's event in the context of `device` (the GPU it is recorded on)."""
    if len(handle) != 64:
        raise DMoEError("an IPC event handle is 64 bytes")
    buf = (ctypes.c_uint8 * 64).from_buffer_copy(handle)
    out = _vp()
    _check(lib_setup().dmoe_ipc_event_open(buf, device, ctypes.byref(out)), "dmoe_ipc_event_open")
    return int(out.value)


def copy_bytes(dst_ptr: int, src_ptr: int, nbytes: int, stream: int) -> None:
    _check(lib().dmoe_copy(dst_ptr, src_ptr, nbytes, stream), "dmoe_copy")


def flag_signal(flag_ptr: int, value: int, stream: int) -> None:
    _check(lib().dmoe_flag_signal(flag_ptr, value, stream), "dmoe_flag_signal")


def flag_wait(flag_ptr: int, value: int, timeout_ns: int, status_ptr: int, stream: int) -> None:
    _check(lib().dmoe_flag_wait(flag_ptr, value, timeout_ns, status_ptr, stream), "dmoe_flag_wait")


# ----------------------------------------------------------------------------- expert-parallel exchange
def ep_flags_bytes() -> int:
    return int(lib().dmoe_ep_flags_bytes())


def ep_counts_bytes(n_inst: int) -> int:
    return int(lib().dmoe_ep_counts_bytes(int(n_inst)))


def ep_window(world: int, rank: int, flags: Sequence[int], counts: Sequence[int], recv: Sequence[int],
              back: Sequence[int], rows: Sequence[int]) -> EpWindow:
    w = EpWindow()
    w.world, w.rank = int(world), int(rank)
    for g in range(world):
        w.flags[g], w.counts[g], w.recv[g], w.back[g], w.rows[g] = flags[g], counts[g], recv[g], back[g], rows[g]
    return w


def ep_plan(win: EpWindow, counts_e: Optional[torch.Tensor], E: int, n_inst: int, policy: int, table, cap: int,
            timeout_ns: int, out, stream: Optional[int] = None) -> None:
    """Count exchange and placement (advances the window's epoch counter).  table: (alive_n,
    alive_inst, inst_rank, inst_slot, inst_first) int32 device tensors; out: (part_n,
    part_inst, part_start, dest_off, seg_expert, seg_end) int32 device tensors."""
    alive_n, alive_inst, inst_rank, inst_slot, inst_first = table
    part_n, part_inst, part_start, dest_off, seg_expert, seg_end = out
    dev = alive_n.device
    st = stream if stream is not None else _stream(dev)
    tm = _Timed("ep_plan", st, dev)
    rc = lib().dmoe_ep_plan(ctypes.byref(win), _ptr(counts_e), E, n_inst, policy, alive_n.data_ptr(),
                            alive_inst.data_ptr(), inst_rank.data_ptr(), inst_slot.data_ptr(), inst_first.data_ptr(),
                            int(cap), int(timeout_ns), part_n.data_ptr(), part_inst.data_ptr(),
                            part_start.data_ptr(), dest_off.data_ptr(), seg_expert.data_ptr(), seg_end.data_ptr(),
                            scratch.status(dev).data_ptr(), st)
    _check(rc, "dmoe_ep_plan")
    tm.done()


def ep_dispatch(win: EpWindow, x: torch.Tensor, T: int, k: int, E: int, offsets: Optional[torch.Tensor],
                perm_token: Optional[torch.Tensor], perm_slot: Optional[torch.Tensor], placement,
                inst_rank: torch.Tensor, cap: int, ret: torch.Tensor, done: torch.Tensor,
                stream: Optional[int] = None) -> None:
    """Gather rows (and their return addresses) into their receivers' windows (peer stores)
    and raise the data flags.  placement: (part_n, part_inst, part_start, dest_off) from
    :func:`ep_plan`."""
    part_n, part_inst, part_start, dest_off = placement
    dev = inst_rank.device
    st = stream if stream is not None else _stream(dev)
    tm = _Timed("ep_dispatch", st, dev)
    rc = lib().dmoe_ep_dispatch(ctypes.byref(win), _ptr(x), x.shape[-1] * x.element_size(), T, k, E, _ptr(offsets),
                                _ptr(perm_token), _ptr(perm_slot), part_n.data_ptr(), part_inst.data_ptr(),
                                part_start.data_ptr(),
                                inst_rank.data_ptr(), dest_off.data_ptr(), int(cap), ret.data_ptr(), done.data_ptr(),
                                scratch.status(dev).data_ptr(), st)
    _check(rc, "dmoe_ep_dispatch")
    tm.done()


def ep_expert_mlp(win: EpWindow, w_gate: torch.Tensor, w_up: torch.Tensor, w_down: torch.Tensor,
                  seg_expert: torch.Tensor, seg_end: torch.Tensor, cap: int, act: int,
                  tile_policy: int = TILES_AUTO, work_rows: Optional[float] = None) -> None:
    """The exchange's expert step: grouped MLP over this rank's receive rows, the
    down-projection stored straight into the hosts' return rows.  work_rows: the rows
    computed, if known, for the timing record's FLOPs."""
    dev = _require_cuda(w_gate, w_up, w_down, seg_expert, seg_end)
    E, I, d = w_gate.shape
    dt = dtype_code(w_gate.dtype)
    ws = scratch.get(dev, "mlp", lib().dmoe_grouped_mlp_workspace_size(cap, I, dt))
    tm = _Timed("grouped_gated_mlp", _stream(dev), dev, None if work_rows is None else 6.0 * work_rows * d * I)
    rc = lib().dmoe_ep_expert_mlp(ctypes.byref(win), w_gate.data_ptr(), w_up.data_ptr(), w_down.data_ptr(), E, d, I, dt,
                                  seg_expert.data_ptr(), seg_end.data_ptr(), seg_expert.numel(), int(cap), int(act),
                                  ws.data_ptr(), ws.numel(), scratch.status(dev).data_ptr(), int(tile_policy),
                                  _stream(dev))
    _check(rc, "dmoe_ep_expert_mlp")
    tm.done()


def ep_expert_mlp_fp8(win: EpWindow, experts: Fp8Experts, seg_expert: torch.Tensor, seg_end: torch.Tensor,
                      cap: int, act: int, tile_policy: int = TILES_AUTO, work_rows: Optional[float] = None) -> None:
    """:func:`ep_expert_mlp` for 8-bit receive records (d e4m3 codes + the row's fp32 scale,
    d + 16 bytes) and e4m3 gate/up stacks; the return rows are bf16."""
    dev = _require_cuda(experts.w_down, seg_expert, seg_end)
    E, I, d = experts.wg_q.shape
    ws = scratch.get(dev, "mlp", lib().dmoe_grouped_mlp_workspace_size(cap, I, BF16))
    tm = _Timed("grouped_gated_mlp", _stream(dev), dev, None if work_rows is None else 6.0 * work_rows * d * I)
    rc = lib().dmoe_ep_expert_mlp_fp8(ctypes.byref(win), experts.wg_q.data_ptr(), experts.wg_scale.data_ptr(),
                                      experts.wu_q.data_ptr(), experts.wu_scale.data_ptr(), experts.w_down.data_ptr(),
                                      E, d, I, seg_expert.data_ptr(), seg_end.data_ptr(), seg_expert.numel(), int(cap),
                                      int(act), ws.data_ptr(), ws.numel(), scratch.status(dev).data_ptr(),
                                      int(tile_policy), _stream(dev))
    _check(rc, "dmoe_ep_expert_mlp_fp8")
    tm.done()


def ep_wait(win: EpWindow, kind: int, timeout_ns: int, device: torch.device, stream: Optional[int] = None) -> None:
    st = stream if stream is not None else _stream(device)
    _check(lib().dmoe_ep_wait(ctypes.byref(win), kind, int(timeout_ns), scratch.status(device).data_ptr(), st),
           "dmoe_ep_wait")


def ep_signal(win: EpWindow, kind: int, device: torch.device, stream: Optional[int] = None) -> None:
    st = stream if stream is not None else _stream(device)
    _check(lib().dmoe_ep_signal(ctypes.byref(win), kind, st), "dmoe_ep_signal")


def ep_combine(win: EpWindow, inverse: Optional[torch.Tensor], ret: torch.Tensor, w: Optional[torch.Tensor],
               T: int, k: int, out: torch.Tensor, accumulate: bool = False, stream: Optional[int] = None) -> None:
    dev = out.device
    st = stream if stream is not None else _stream(dev)
    tm = _Timed("ep_combine", st, dev)
    rc = lib().dmoe_ep_combine(ctypes.byref(win), _ptr(inverse), ret.data_ptr(), _ptr(w),
                               dtype_code(w.dtype) if w is not None else F32, T, k, out.shape[-1],
                               dtype_code(out.dtype), int(accumulate), out.data_ptr(), st)
    _check(rc, "dmoe_ep_combine")
    tm.done()


_graph_launches = 0
_graph_lock = threading.Lock()


def count_graph_replay(launches: int) -> None:
    """Account the library kernels of one CUDA-graph replay (captured launches run again
    without passing through the C entry points that count them)."""
    global _graph_launches
    with _graph_lock:
        _graph_launches += int(launches)


def launch_count() -> int:
    """Library kernels launched in this process: direct launches plus graph replays."""
    return int(lib().dmoe_launch_count()) + _graph_launches
