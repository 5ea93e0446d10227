"""Drop-in ``ltc_cuda`` for the LTC ODE solver, backed by libltc_sm100.so (sm_100a).

This module keeps the names and call signatures the reference's ``ltc.py``
imports (``from ltc_cuda import _HAS_CUDA_KERNELS, ltc_cuda_forward``,
``ltc.py:12-16``) and the reference's bridge exposes (``ltc_cuda.py:241-388``):

* ``_HAS_CUDA_KERNELS``  -- True when the library loaded and a CUDA device is present
* ``ltc_cuda_forward(x_seq, state, w_pos, w_erev, mu, sigma, sensory_mu,
  sensory_sigma, sensory_erev, sensory_w_pos, cm_t, gleak_pos, vleak,
  ode_unfolds, epsilon) -> (outputs, state)``  (``ltc_cuda.py:362-388``)
* ``LTCCudaForward``     -- the autograd.Function (``ltc_cuda.py:241-359``): forward
  takes the same 15 inputs plus ``needs_grad``; backward returns 13 gradients
  in input order followed by three ``None``
* ``_cuda_module.ltc_full_forward`` / ``ltc_full_backward`` -- the whole-sequence
  forward/backward calls (``csrc/ltc_kernels.cu:1165``, ``:962``)

Differences from the reference bridge, all internal to this module: parameters
are passed untransposed (no transposed copies are made), the forward saves one
opaque buffer (per-unfold states and reciprocal denominators) instead of the
(T,U,B,H) state stack plus the two sensory stacks, and every kernel runs on
PyTorch's current stream instead of the legacy default stream.

There is no fallback inside this module: on a machine with CUDA, a missing or
unloadable library raises at import; calling ``ltc_cuda_forward`` without CUDA
kernels raises ``RuntimeError``.
"""
from __future__ import annotations

import ctypes
import logging
import os
import threading
from typing import List, Optional, Sequence

import torch

logger = logging.getLogger(__name__)

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("LTC_SM100_LIB", os.path.join(_HERE, "libltc_sm100.so"))

LTC_FLAG_FORCE_WIDE = 1
LTC_FLAG_LEAN_SAVE = 2
LTC_FLAG_SKIP_ZERO_SYNAPSES = 4
LTC_FLAG_SKIP_ZERO_SENSORY = 1 << 24
LTC_LEAN_CHUNK_SHIFT = 8


class LtcDims(ctypes.Structure):
    _fields_ = [("B", ctypes.c_int32), ("T", ctypes.c_int32), ("D", ctypes.c_int32), ("H", ctypes.c_int32),
                ("ode_unfolds", ctypes.c_int32), ("epsilon", ctypes.c_float), ("flags", ctypes.c_int32)]


class LtcParams(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in (
        "w_pos", "w_erev", "mu", "sigma", "sensory_mu", "sensory_sigma", "sensory_erev",
        "sensory_w_pos", "cm_t", "gleak_pos", "vleak")]


class LtcGrads(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in (
        "x_seq", "state", "w_pos", "w_erev", "mu", "sigma", "sensory_mu", "sensory_sigma",
        "sensory_erev", "sensory_w_pos", "cm_t", "gleak_pos", "vleak")]


class LtcPlan(ctypes.Structure):
    _fields_ = [("saved_bytes", ctypes.c_size_t), ("fwd_workspace_bytes", ctypes.c_size_t),
                ("bwd_workspace_bytes", ctypes.c_size_t), ("wide", ctypes.c_int32),
                ("padded_h", ctypes.c_int32), ("fwd_ctas", ctypes.c_int32), ("bwd_ctas", ctypes.c_int32),
                ("lean_chunk_steps", ctypes.c_int32)]


# Exported symbols and their C signatures (include/ltc_sm100.h).
EXPORTS = {
    "ltc_plan": (ctypes.c_int, [ctypes.POINTER(LtcDims), ctypes.POINTER(LtcPlan)]),
    "ltc_forward": (ctypes.c_int, [ctypes.POINTER(LtcDims), ctypes.POINTER(LtcParams), ctypes.c_void_p,
                                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                   ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "ltc_backward": (ctypes.c_int, [ctypes.POINTER(LtcDims), ctypes.POINTER(LtcParams), ctypes.c_void_p,
                                    ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_int64),
                                    ctypes.c_void_p, ctypes.POINTER(LtcGrads), ctypes.c_void_p,
                                    ctypes.c_size_t, ctypes.c_void_p]),
    "ltc_preamble_forward": (ctypes.c_int, [ctypes.c_int64, ctypes.c_int32, ctypes.c_float] + [ctypes.c_void_p] * 8),
    "ltc_preamble_workspace_bytes": (ctypes.c_size_t, [ctypes.c_int64, ctypes.c_int32]),
    "ltc_preamble_backward": (ctypes.c_int, [ctypes.c_int64, ctypes.c_int32] + [ctypes.c_void_p] * 12
                              + [ctypes.c_size_t, ctypes.c_void_p]),
    "ltc_forward_noalloc": (ctypes.c_int, [ctypes.POINTER(LtcDims), ctypes.POINTER(LtcParams)]
                            + [ctypes.c_void_p] * 5),
    "ltc_step_workspace_bytes": (ctypes.c_int, [ctypes.POINTER(LtcDims), ctypes.c_int,
                                                 ctypes.POINTER(ctypes.c_size_t)]),
    "ltc_step_sensory_forward": (ctypes.c_int, [ctypes.POINTER(LtcDims), ctypes.POINTER(LtcParams)]
                                 + [ctypes.c_void_p] * 4 + [ctypes.c_size_t, ctypes.c_void_p]),
    "ltc_step_unfold_forward": (ctypes.c_int, [ctypes.POINTER(LtcDims), ctypes.POINTER(LtcParams)]
                                + [ctypes.c_void_p] * 6 + [ctypes.c_size_t, ctypes.c_void_p]),
    "ltc_step_sensory_backward": (ctypes.c_int, [ctypes.POINTER(LtcDims), ctypes.POINTER(LtcParams)]
                                  + [ctypes.c_void_p] * 9 + [ctypes.c_size_t, ctypes.c_void_p]),
    "ltc_step_unfold_backward": (ctypes.c_int, [ctypes.POINTER(LtcDims), ctypes.POINTER(LtcParams)]
                                 + [ctypes.c_void_p] * 15 + [ctypes.c_size_t, ctypes.c_void_p]),
    "ltc_timing_enable": (ctypes.c_int, [ctypes.c_int]),
    "ltc_timing_collect": (ctypes.c_int, [ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_int32),
                                          ctypes.c_int]),
    "ltc_launch_count": (ctypes.c_int64, []),
    "ltc_wait_timeouts": (ctypes.c_int, []),
    "ltc_last_error": (ctypes.c_char_p, []),
    "ltc_version": (ctypes.c_int, []),
}


def load_library(path: str = LIB_PATH) -> ctypes.CDLL:
    lib = ctypes.CDLL(path)
    for name, (res, args) in EXPORTS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


_lib: Optional[ctypes.CDLL] = None
_load_error: Optional[str] = None
try:
    _lib = load_library()
except OSError as exc:  # library not built
    _load_error = str(exc)

if _lib is None and torch.cuda.is_available():
    raise RuntimeError(
        f"ltc_cuda: CUDA is available but {LIB_PATH} could not be loaded ({_load_error}); "
        "build it with `python ltc-cuda_b200/build.py` (there is no CPU/TorchScript fallback)")

_HAS_CUDA_KERNELS: bool = _lib is not None and torch.cuda.is_available()


def _check(status: int, what: str) -> None:
    if status != 0:
        msg = _lib.ltc_last_error().decode(errors="replace") if _lib is not None else "library not loaded"
        raise RuntimeError(f"ltc_cuda.{what} failed: {msg}")


def _require_kernels() -> ctypes.CDLL:
    if not _HAS_CUDA_KERNELS:
        raise RuntimeError("ltc_cuda: CUDA kernels unavailable "
                           f"(library: {_load_error or 'loaded'}, cuda: {torch.cuda.is_available()})")
    return _lib


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _as_f32(t: torch.Tensor, device: torch.device, name: str) -> torch.Tensor:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a tensor")
    if t.device != device:
        raise ValueError(f"{name} is on {t.device}, expected {device}")
    if t.dtype != torch.float32:
        raise TypeError(f"{name} must be float32 (got {t.dtype})")
    return t.contiguous()


def make_dims(B: int, T: int, D: int, H: int, ode_unfolds: int, epsilon: float, flags: int = 0) -> LtcDims:
    return LtcDims(int(B), int(T), int(D), int(H), int(ode_unfolds), float(epsilon), int(flags))


def plan(dims: LtcDims) -> LtcPlan:
    lib = _require_kernels()
    p = LtcPlan()
    _check(lib.ltc_plan(ctypes.byref(dims), ctypes.byref(p)), "ltc_plan")
    return p


_flags = 0


def set_force_wide(on: bool) -> None:
    """Route every call through the streamed wide-H kernels (testing the second path)."""
    global _flags
    _flags = (_flags | LTC_FLAG_FORCE_WIDE) if on else (_flags & ~LTC_FLAG_FORCE_WIDE)


def set_lean_save(on: bool, chunk_steps: int = 0) -> None:
    """Memory-lean training: the forward keeps only the state at each step boundary
    and the backward recomputes the unfolds segment by segment (``chunk_steps`` steps
    per segment; 0 = sized by the library).  Applies to forwards run afterwards; a
    forward's own mode is remembered for its backward."""
    global _flags
    _flags &= ~(LTC_FLAG_LEAN_SAVE | (0xFFFF << LTC_LEAN_CHUNK_SHIFT))
    if on:
        _flags |= LTC_FLAG_LEAN_SAVE | ((int(chunk_steps) & 0xFFFF) << LTC_LEAN_CHUNK_SHIFT)


_call_flags = threading.local()


class skip_zero_synapses:
    """Context manager: solver calls made inside it (forward, and the backward of those
    forwards) skip recurrent synapses whose ``w_pos`` and ``w_erev`` are both zero
    (``LTC_FLAG_SKIP_ZERO_SYNAPSES``).  The solver's gradients of ``w_pos``, ``w_erev``,
    ``mu`` and ``sigma`` are then zero at those positions instead of the dense values --
    use it only where those entries are discarded, as when ``w_pos = softplus(w) * mask``
    (the module's transforms).  Other outputs are unchanged.

    ``sensory=True`` (with ``on``) also skips the sensory synapses whose
    ``sensory_w_pos`` is zero in the sensory backward (``LTC_FLAG_SKIP_ZERO_SENSORY``,
    any H): the four sensory gradients are then zero at those positions -- again only
    for callers that discard them, as ``sensory_w_pos = softplus(w) * mask`` does.
    Check the pattern with :func:`skip_zero_sensory_fits` first."""

    def __init__(self, on: bool = True, sensory: bool = False):
        self.on = bool(on)
        self.sensory = bool(on and sensory)

    def __enter__(self):
        self.prev = getattr(_call_flags, "extra", 0)
        both = LTC_FLAG_SKIP_ZERO_SYNAPSES | LTC_FLAG_SKIP_ZERO_SENSORY
        flags = self.prev & ~both
        if self.on:
            flags |= LTC_FLAG_SKIP_ZERO_SYNAPSES
        if self.sensory:
            flags |= LTC_FLAG_SKIP_ZERO_SENSORY
        _call_flags.extra = flags
        return self

    def __exit__(self, *exc):
        _call_flags.extra = self.prev
        return False


# Capacity of the synapse-skipping kernels.  32 < H <= 64: at most this many nonzero
# synapses per neuron (incoming and outgoing); H <= 32: any mask.  128 < H <= 512
# (HP = 256 or 512 padded neurons, 8 blocks of HP/8): at most 8192 nonzero synapses
# enter each block, and inside each block the rows, ranked by outgoing count and
# paired c-th heaviest with c-th lightest in warps of 4 pairs, need
# 4*ceil(max ceil(heavy/8)/4) + 4*ceil(max ceil(light/8)/4) <= 32 slots per warp.
# 64 < H <= 128 runs dense kernels (the flag is ignored).  A call beyond the capacity
# gets NaN outputs from the kernels, so callers check first.
SKIP_MAX_SYNAPSES_PER_NEURON = 48
SKIP_WIDE_MAX_PER_BLOCK = 8192
SKIP_WIDE_SLOTS_PER_LANE = 32


def _wide_fits(nz: torch.Tensor) -> bool:
    H = nz.shape[0]
    HP = 256 if H <= 256 else 512
    NEUR = HP // 8
    pad = torch.zeros(HP, HP, dtype=torch.bool, device=nz.device)
    pad[:H, :H] = nz
    if int(pad.sum(0).view(8, NEUR).sum(1).max().item()) > SKIP_WIDE_MAX_PER_BLOCK:
        return False
    rows = pad.sum(1).view(8, NEUR).sort(dim=1, descending=True).values  # per block, heaviest first
    heavy = (rows[:, :NEUR // 2] + 7) // 8
    light = (rows.flip(1)[:, :NEUR // 2] + 7) // 8
    k1 = (heavy.view(8, -1, 4).max(2).values + 3) // 4 * 4
    k2 = (light.view(8, -1, 4).max(2).values + 3) // 4 * 4
    return int((k1 + k2).max().item()) <= SKIP_WIDE_SLOTS_PER_LANE


def skip_zero_synapses_fits(mask: torch.Tensor) -> bool:
    """True when the (H, H) nonzero pattern ``mask`` fits the synapse-skipping kernels."""
    H = mask.shape[0]
    nz = mask != 0
    if H <= 32 or 64 < H <= 128:
        return True
    if H <= 64:
        return int(torch.maximum(nz.sum(0).max(), nz.sum(1).max()).item()) <= SKIP_MAX_SYNAPSES_PER_NEURON
    return _wide_fits(nz)


def skip_zero_sensory_fits(smask: torch.Tensor) -> bool:
    """True when the (D, H) sensory pattern fits the sensory backward's skipping kernel:
    any pattern for H <= 32; otherwise at most 48 nonzero synapses per input and per
    column inside every 64 x 64 block (64 consecutive inputs x 64 consecutive columns)."""
    D, H = smask.shape
    if H <= 32:
        return True
    nz = (smask != 0)
    for d0 in range(0, D, 64):
        for q0 in range(0, H, 64):
            blk = nz[d0:d0 + 64, q0:q0 + 64]
            if int(blk.sum(1).max().item()) > SKIP_MAX_SYNAPSES_PER_NEURON or \
                    int(blk.sum(0).max().item()) > SKIP_MAX_SYNAPSES_PER_NEURON:
                return False
    return True


def _call_flags_now() -> int:
    return _flags | getattr(_call_flags, "extra", 0)


KERNEL_NAMES = ("pack_fwd", "sensory_fwd", "recurrent_fwd", "pack_bwd", "recurrent_bwd", "sensory_bwd",
                "finish", "preamble_fwd", "preamble_bwd")


def timing_enable(on: bool) -> None:
    """Bracket every library launch with CUDA events on its own stream (see ltc_timing_enable)."""
    _check(_require_kernels().ltc_timing_enable(1 if on else 0), "ltc_timing_enable")


def timing_collect() -> dict:
    """{kernel name: (total ms, launches)} since timing was enabled or last collected."""
    lib = _require_kernels()
    n = len(KERNEL_NAMES)
    ms = (ctypes.c_double * n)()
    cnt = (ctypes.c_int32 * n)()
    _check(lib.ltc_timing_collect(ms, cnt, n), "ltc_timing_collect")
    return {k: (ms[i], cnt[i]) for i, k in enumerate(KERNEL_NAMES)}


def launch_count() -> int:
    return int(_require_kernels().ltc_launch_count())


def wait_timeouts() -> int:
    """Bounded in-kernel cluster waits that expired on the current device (0 when healthy)."""
    n = int(_require_kernels().ltc_wait_timeouts())
    if n < 0:
        raise RuntimeError("ltc_wait_timeouts: " + _require_kernels().ltc_last_error().decode())
    return n


_CHECK_WAITS = [False, 0]


def set_check_waits(on: bool) -> None:
    """Opt-in health check: when on, every backward pass ends by reading the device's
    expired-wait counter (one small device-to-host read, so it synchronises the device)
    and raises ``RuntimeError`` if a bounded in-kernel wait expired since the previous
    check -- such a launch finished without its peer data and its results are invalid.
    Off by default; callers that leave it off should poll :func:`wait_timeouts` at a
    step boundary they already synchronise on."""
    _CHECK_WAITS[0] = bool(on)
    _CHECK_WAITS[1] = wait_timeouts() if on else 0


def _check_waits_after(where: str) -> None:
    n = wait_timeouts()
    if n != _CHECK_WAITS[1]:
        _CHECK_WAITS[1] = n
        raise RuntimeError(f"{where}: {n} bounded in-kernel wait(s) expired on this device; results are invalid")


def _params_struct(ts: Sequence[torch.Tensor]) -> LtcParams:
    return LtcParams(*[t.data_ptr() for t in ts])


class _CudaModule:
    """Whole-sequence calls with the reference's names (``csrc/ltc_kernels.cu:1307-1314``)."""

    @staticmethod
    def ltc_full_forward(x_seq, state, w_pos, w_erev, mu, sigma, sensory_mu, sensory_sigma, sensory_erev,
                         sensory_w_pos, cm_t, gleak_pos, vleak, ode_unfolds: int, epsilon: float,
                         save_intermediates: bool) -> List[torch.Tensor]:
        """Returns [outputs (B,T,H), final state (B,H)] (+ [saved] when save_intermediates)."""
        lib = _require_kernels()
        dev = x_seq.device
        x = _as_f32(x_seq, dev, "x_seq")
        B, T, D = x.shape
        H = state.shape[1]
        h0 = _as_f32(state, dev, "state")
        params = [_as_f32(t, dev, n) for t, n in zip(
            (w_pos, w_erev, mu, sigma, sensory_mu, sensory_sigma, sensory_erev, sensory_w_pos,
             cm_t, gleak_pos, vleak),
            ("w_pos", "w_erev", "mu", "sigma", "sensory_mu", "sensory_sigma", "sensory_erev",
             "sensory_w_pos", "cm_t", "gleak_pos", "vleak"))]
        _check_shapes(B, T, D, H, params)
        outputs = torch.empty(B, T, H, device=dev, dtype=torch.float32)
        if B == 0 or T == 0 or int(ode_unfolds) <= 0:
            return _degenerate_forward(x, h0, outputs, save_intermediates)
        dims = make_dims(B, T, D, H, ode_unfolds, epsilon, _call_flags_now())
        with torch.cuda.device(dev):
            pl = plan(dims)
            h_final = torch.empty(B, H, device=dev, dtype=torch.float32)
            saved = torch.empty(pl.saved_bytes, device=dev, dtype=torch.uint8) if save_intermediates else None
            ws = torch.empty(pl.fwd_workspace_bytes, device=dev, dtype=torch.uint8)
            stream = torch.cuda.current_stream(dev).cuda_stream
            _check(lib.ltc_forward(ctypes.byref(dims), ctypes.byref(_params_struct(params)), x.data_ptr(),
                                   h0.data_ptr(), outputs.data_ptr(), h_final.data_ptr(), _ptr(saved),
                                   ws.data_ptr(), pl.fwd_workspace_bytes, stream), "ltc_full_forward")
        if saved is not None:
            saved._ltc_flags = dims.flags  # the backward must read it with the same layout
        return [outputs, h_final, saved] if save_intermediates else [outputs, h_final]

    @staticmethod
    def ltc_full_backward(x_seq, state, w_pos, w_erev, mu, sigma, sensory_mu, sensory_sigma, sensory_erev,
                          sensory_w_pos, cm_t, gleak_pos, vleak, saved, grad_outputs, grad_final_state,
                          ode_unfolds: int, epsilon: float, has_grad_state: bool) -> List[torch.Tensor]:
        """13 gradients in the order of the forward inputs (``ltc_cuda.py:342-355``)."""
        lib = _require_kernels()
        dev = x_seq.device
        x = _as_f32(x_seq, dev, "x_seq")
        B, T, D = x.shape
        H = state.shape[1]
        params = [_as_f32(t, dev, "param") for t in (w_pos, w_erev, mu, sigma, sensory_mu, sensory_sigma,
                                                     sensory_erev, sensory_w_pos, cm_t, gleak_pos, vleak)]
        if grad_outputs is None:
            grad_outputs = torch.zeros(1, device=dev, dtype=torch.float32).expand(B, T, H)
        elif grad_outputs.dtype != torch.float32:
            grad_outputs = grad_outputs.float()
        gs = None
        if has_grad_state and grad_final_state is not None:
            gs = _as_f32(grad_final_state, dev, "grad_final_state")
        grads = [torch.empty(B, T, D, device=dev), torch.empty(B, H, device=dev)] + \
                [torch.empty_like(p) for p in params]
        dims = make_dims(B, T, D, H, ode_unfolds, epsilon, getattr(saved, "_ltc_flags", _flags))
        strides = (ctypes.c_int64 * 3)(*grad_outputs.stride())
        with torch.cuda.device(dev):
            pl = plan(dims)
            ws = torch.empty(pl.bwd_workspace_bytes, device=dev, dtype=torch.uint8)
            stream = torch.cuda.current_stream(dev).cuda_stream
            _check(lib.ltc_backward(ctypes.byref(dims), ctypes.byref(_params_struct(params)), x.data_ptr(),
                                    saved.data_ptr(), grad_outputs.data_ptr(), strides, _ptr(gs),
                                    ctypes.byref(LtcGrads(*[g.data_ptr() for g in grads])), ws.data_ptr(),
                                    pl.bwd_workspace_bytes, stream), "ltc_full_backward")
        return grads


    # ---- step-level calls with the reference's names (csrc/ltc_kernels.cu:1308-1311) ----

    @staticmethod
    def _step(kind, dims, fn_name, params, ptrs, dev):
        lib = _require_kernels()
        nbytes = ctypes.c_size_t(0)
        with torch.cuda.device(dev):
            _check(lib.ltc_step_workspace_bytes(ctypes.byref(dims), kind, ctypes.byref(nbytes)), fn_name)
            ws = torch.empty(max(1, nbytes.value), dtype=torch.uint8, device=dev)
            st = torch.cuda.current_stream(dev).cuda_stream
            _check(getattr(lib, fn_name)(ctypes.byref(dims), ctypes.byref(params), *ptrs, ws.data_ptr(),
                                         nbytes.value, st), fn_name)

    @staticmethod
    def ltc_sensory_fwd(inputs, sensory_sigma, sensory_mu, sensory_w_pos, sensory_erev):
        """(B,D) inputs of one step -> [w_num_sensory, w_den_sensory] (B,H)."""
        dev = inputs.device
        x = _as_f32(inputs, dev, "inputs")
        B, D = x.shape
        H = sensory_sigma.shape[1]
        ps = {n: _as_f32(t, dev, n) for n, t in (("sensory_sigma", sensory_sigma), ("sensory_mu", sensory_mu),
                                                  ("sensory_w_pos", sensory_w_pos), ("sensory_erev", sensory_erev))}
        params = LtcParams(sensory_mu=ps["sensory_mu"].data_ptr(), sensory_sigma=ps["sensory_sigma"].data_ptr(),
                           sensory_erev=ps["sensory_erev"].data_ptr(), sensory_w_pos=ps["sensory_w_pos"].data_ptr())
        wn = torch.empty(B, H, device=dev)
        wd = torch.empty(B, H, device=dev)
        _CudaModule._step(0, make_dims(B, 1, D, H, 1, 0.0, _flags), "ltc_step_sensory_forward", params,
                          [x.data_ptr(), wn.data_ptr(), wd.data_ptr()], dev)
        return [wn, wd]

    @staticmethod
    def _rec_params(dev, w_pos, w_erev, mu, sigma, cm_t, gleak_pos, vleak):
        ts = [_as_f32(t, dev, "param") for t in (w_pos, w_erev, mu, sigma, cm_t, gleak_pos, vleak)]
        return ts, LtcParams(w_pos=ts[0].data_ptr(), w_erev=ts[1].data_ptr(), mu=ts[2].data_ptr(),
                             sigma=ts[3].data_ptr(), cm_t=ts[4].data_ptr(), gleak_pos=ts[5].data_ptr(),
                             vleak=ts[6].data_ptr())

    @staticmethod
    def ltc_ode_unfold_fwd(state, w_pos, w_erev, mu, sigma, w_num_sensory, w_den_sensory, cm_t, gleak_pos, vleak,
                           ode_unfolds: int, epsilon: float, save_intermediates: bool):
        """One step's unfolds -> [state (B,H), v_buffer (U,B,H) or an empty tensor]."""
        dev = state.device
        st_ = _as_f32(state, dev, "state")
        B, H = st_.shape
        ts, params = _CudaModule._rec_params(dev, w_pos, w_erev, mu, sigma, cm_t, gleak_pos, vleak)
        wn = _as_f32(w_num_sensory, dev, "w_num_sensory")
        wd = _as_f32(w_den_sensory, dev, "w_den_sensory")
        out = torch.empty(B, H, device=dev)
        vb = torch.empty(int(ode_unfolds), B, H, device=dev) if save_intermediates else None
        _CudaModule._step(1, make_dims(B, 1, 1, H, ode_unfolds, epsilon, _flags), "ltc_step_unfold_forward",
                          params, [st_.data_ptr(), wn.data_ptr(), wd.data_ptr(), out.data_ptr(), _ptr(vb)], dev)
        return [out, vb if vb is not None else torch.empty(0, device=dev)]

    @staticmethod
    def ltc_sensory_bwd(grad_w_num, grad_w_den, inputs, sensory_sigma, sensory_mu, sensory_w_pos, sensory_erev):
        """-> [grad_inputs (B,D), grad sensory_sigma, sensory_mu, sensory_w_pos, sensory_erev (D,H)]."""
        dev = inputs.device
        x = _as_f32(inputs, dev, "inputs")
        B, D = x.shape
        H = sensory_sigma.shape[1]
        ps = [_as_f32(t, dev, "param") for t in (sensory_sigma, sensory_mu, sensory_w_pos, sensory_erev)]
        params = LtcParams(sensory_sigma=ps[0].data_ptr(), sensory_mu=ps[1].data_ptr(),
                           sensory_w_pos=ps[2].data_ptr(), sensory_erev=ps[3].data_ptr())
        gn = _as_f32(grad_w_num, dev, "grad_w_num")
        gd = _as_f32(grad_w_den, dev, "grad_w_den")
        gx = torch.empty(B, D, device=dev)
        outs = [torch.empty(D, H, device=dev) for _ in range(4)]
        _CudaModule._step(2, make_dims(B, 1, D, H, 1, 0.0, _flags), "ltc_step_sensory_backward", params,
                          [gn.data_ptr(), gd.data_ptr(), x.data_ptr(), gx.data_ptr()] + [o.data_ptr() for o in outs],
                          dev)
        return [gx] + outs

    @staticmethod
    def ltc_ode_unfold_bwd(v_buffer, w_pos, w_erev, mu, sigma, w_num_sensory, w_den_sensory, cm_t, gleak_pos, vleak,
                           grad_output, ode_unfolds: int, epsilon: float):
        """-> [grad_v, grad_w_num, grad_w_den (B,H), grad w_pos, w_erev, mu, sigma (H,H), grad cm, gleak, vleak (H)]."""
        dev = v_buffer.device
        vb = _as_f32(v_buffer, dev, "v_buffer")
        _, B, H = vb.shape
        ts, params = _CudaModule._rec_params(dev, w_pos, w_erev, mu, sigma, cm_t, gleak_pos, vleak)
        wn = _as_f32(w_num_sensory, dev, "w_num_sensory")
        wd = _as_f32(w_den_sensory, dev, "w_den_sensory")
        go = _as_f32(grad_output, dev, "grad_output")
        outs = [torch.empty(B, H, device=dev) for _ in range(3)] + [torch.empty(H, H, device=dev) for _ in range(4)] \
            + [torch.empty(H, device=dev) for _ in range(3)]
        _CudaModule._step(3, make_dims(B, 1, 1, H, ode_unfolds, epsilon, _flags), "ltc_step_unfold_backward",
                          params, [vb.data_ptr(), wn.data_ptr(), wd.data_ptr(), go.data_ptr()]
                          + [o.data_ptr() for o in outs], dev)
        return outs


_cuda_module = _CudaModule()


def _check_shapes(B, T, D, H, params):
    expect = [(H, H)] * 4 + [(D, H)] * 4 + [(H,)] * 3
    names = ("w_pos", "w_erev", "mu", "sigma", "sensory_mu", "sensory_sigma", "sensory_erev",
             "sensory_w_pos", "cm_t", "gleak_pos", "vleak")
    for t, e, n in zip(params, expect, names):
        if tuple(t.shape) != e:
            raise ValueError(f"{n} has shape {tuple(t.shape)}, expected {e}")


def _degenerate_forward(x, h0, outputs, save_intermediates):
    """B == 0, T == 0 or no unfolds: the state passes through unchanged (``ltc.py:50-63,96-104``)."""
    B, T = x.shape[:2]
    if T > 0 and B > 0:
        outputs.copy_(h0.unsqueeze(1).expand(B, T, h0.shape[1]))
    h = h0.clone()
    return [outputs, h, torch.empty(0, dtype=torch.uint8, device=x.device)] if save_intermediates else [outputs, h]


class LTCCudaForward(torch.autograd.Function):
    """Autograd bridge with the reference's argument order (``ltc_cuda.py:241-359``)."""

    @staticmethod
    def forward(ctx, x_seq, state, w_pos, w_erev, mu, sigma, sensory_mu, sensory_sigma, sensory_erev,
                sensory_w_pos, cm_t, gleak_pos, vleak, ode_unfolds: int, epsilon: float, needs_grad: bool):
        res = _cuda_module.ltc_full_forward(x_seq, state, w_pos, w_erev, mu, sigma, sensory_mu, sensory_sigma,
                                            sensory_erev, sensory_w_pos, cm_t, gleak_pos, vleak,
                                            ode_unfolds, epsilon, needs_grad)
        outputs, h = res[0], res[1]
        if needs_grad:
            ctx.save_for_backward(x_seq, state, w_pos, w_erev, mu, sigma, sensory_mu, sensory_sigma,
                                  sensory_erev, sensory_w_pos, cm_t, gleak_pos, vleak, res[2])
        ctx.ode_unfolds = int(ode_unfolds)
        ctx.epsilon = float(epsilon)
        ctx.set_materialize_grads(False)
        return outputs, h

    @staticmethod
    def backward(ctx, grad_outputs, grad_state):
        saved = ctx.saved_tensors
        if not saved:
            raise RuntimeError("LTCCudaForward.backward: forward ran with needs_grad=False")
        (x_seq, state, w_pos, w_erev, mu, sigma, smu, ssig, serev, sw, cm_t, gleak_pos, vleak, buf) = saved
        B, T, _ = x_seq.shape
        H = state.shape[1]
        if B == 0 or T == 0 or ctx.ode_unfolds <= 0:
            return _degenerate_backward(x_seq, state, w_pos, w_erev, mu, sigma, smu, ssig, serev, sw, cm_t,
                                        gleak_pos, vleak, grad_outputs, grad_state)
        g = _cuda_module.ltc_full_backward(x_seq, state, w_pos, w_erev, mu, sigma, smu, ssig, serev, sw, cm_t,
                                           gleak_pos, vleak, buf, grad_outputs, grad_state, ctx.ode_unfolds,
                                           ctx.epsilon, grad_state is not None)
        if _CHECK_WAITS[0]:
            _check_waits_after("LTCCudaForward.backward")
        return (*g, None, None, None)


def _degenerate_backward(x_seq, state, *rest):
    params, (grad_outputs, grad_state) = rest[:11], rest[11:]
    gh = torch.zeros_like(state)
    if grad_state is not None:
        gh = gh + grad_state
    if grad_outputs is not None and grad_outputs.numel() > 0:
        gh = gh + grad_outputs.sum(dim=1)
    return (torch.zeros_like(x_seq), gh, *[torch.zeros_like(p) for p in params], None, None, None)


def ltc_cuda_forward(x_seq, state, w_pos, w_erev, mu, sigma, sensory_mu, sensory_sigma, sensory_erev,
                     sensory_w_pos, cm_t, gleak_pos, vleak, ode_unfolds: int, epsilon: float):
    """Entry point used by ``ltc.py:300-307``: grad mode is read here, outside the Function."""
    _require_kernels()
    needs_grad = torch.is_grad_enabled()
    return LTCCudaForward.apply(x_seq, state, w_pos, w_erev, mu, sigma, sensory_mu, sensory_sigma,
                                sensory_erev, sensory_w_pos, cm_t, gleak_pos, vleak, ode_unfolds, epsilon,
                                needs_grad)


# ---------------------------------------------------------------------------
# Fused module preamble: LayerNorm + input affine map (ltc.py:259, ltc.py:266)
# ---------------------------------------------------------------------------
PREAMBLE_MAX_D = 1024


class LtcPreamble(torch.autograd.Function):
    """y = (LayerNorm(x; ln_w, ln_b, eps) * in_w + in_b) in one sm_100a kernel per direction."""

    @staticmethod
    def forward(ctx, x, ln_w, ln_b, in_w, in_b, eps: float):
        lib = _require_kernels()
        dev = x.device
        xc = _as_f32(x, dev, "x")
        D = xc.shape[-1]
        rows = xc.numel() // D
        params = [_as_f32(t, dev, n) for t, n in ((ln_w, "ln_w"), (ln_b, "ln_b"), (in_w, "in_w"), (in_b, "in_b"))]
        y = torch.empty_like(xc)
        stats = torch.empty(rows, 2, device=dev, dtype=torch.float32)
        with torch.cuda.device(dev):
            st = torch.cuda.current_stream(dev).cuda_stream
            _check(lib.ltc_preamble_forward(rows, D, float(eps), xc.data_ptr(), *[t.data_ptr() for t in params],
                                            y.data_ptr(), stats.data_ptr(), st), "ltc_preamble_forward")
        ctx.save_for_backward(xc, params[0], params[1], params[2], stats)
        return y

    @staticmethod
    def backward(ctx, dy):
        lib = _require_kernels()
        xc, ln_w, ln_b, in_w, stats = ctx.saved_tensors
        dev = xc.device
        D = xc.shape[-1]
        rows = xc.numel() // D
        dyc = dy.to(torch.float32).contiguous()
        dx = torch.empty_like(xc)
        grads = [torch.empty(D, device=dev, dtype=torch.float32) for _ in range(4)]  # ln_w, ln_b, in_w, in_b
        with torch.cuda.device(dev):
            nbytes = lib.ltc_preamble_workspace_bytes(rows, D)
            ws = torch.empty(max(1, nbytes), dtype=torch.uint8, device=dev)
            st = torch.cuda.current_stream(dev).cuda_stream
            _check(lib.ltc_preamble_backward(rows, D, xc.data_ptr(), dyc.data_ptr(), ln_w.data_ptr(),
                                             ln_b.data_ptr(), in_w.data_ptr(), stats.data_ptr(), dx.data_ptr(),
                                             *[g.data_ptr() for g in grads], ws.data_ptr(), nbytes, st),
                   "ltc_preamble_backward")
        return dx, grads[0], grads[1], grads[2], grads[3], None


def ltc_preamble(x, ln_w, ln_b, in_w, in_b, eps: float):
    """Fused LayerNorm + affine map over the last dimension (D <= 1024)."""
    return LtcPreamble.apply(x, ln_w, ln_b, in_w, in_b, eps)
