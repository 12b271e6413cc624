"""torch-facing wrappers of the sm_100a kernels (one function per C ABI stage).

Every function takes CUDA tensors, launches on the current torch stream and
returns new tensors; nothing synchronises with the host.  A batch of
"cells" is a list of same-shape, same-dtype contiguous tensors (one layer's
K and V, or many layers): one launch covers the whole batch.
"""

from __future__ import annotations

import ctypes
from typing import Sequence

import torch

from kvcompress_b200._native import KVC, check, lib, ptr_array

__all__ = [
    "DTYPE_CODE",
    "Cells",
    "DecodePlan",
    "apply_basis",
    "cells",
    "compress",
    "cast",
    "core",
    "decompress",
    "decompress_noalloc",
    "gram",
    "project_feature",
    "residual_quant",
    "residual_stats",
    "sketch_solve",
    "split",
    "workspace",
]

DTYPE_CODE = {torch.float32: KVC.F32, torch.float16: KVC.F16, torch.bfloat16: KVC.BF16,
              torch.float64: KVC.F64}
if hasattr(torch, "float8_e4m3fn"):
    DTYPE_CODE[torch.float8_e4m3fn] = KVC.FP8E4M3

_WS: dict[tuple[int, int], torch.Tensor] = {}

# Optional launch log for the benchmark: (stage, start event, end event,
# kernel launches, algorithmic bytes) per C ABI call on the current stream.
_TRACE: list | None = None
_TRACE_STAGES: frozenset | None = None  # stages to record (None: every stage)


def trace_start(stages=None) -> None:
    """Record CUDA events around every stage launched from now on, or only
    around the named ``stages`` (each recorded event pair costs the stream a
    little time, so a timed run records only the stages it reports)."""
    global _TRACE, _TRACE_STAGES
    _TRACE = []
    _TRACE_STAGES = None if stages is None else frozenset(stages)


def _traced(name: str) -> bool:
    return _TRACE is not None and (_TRACE_STAGES is None or name in _TRACE_STAGES)


def trace_stop() -> list:
    """Stop recording and return the log."""
    global _TRACE, _TRACE_STAGES
    log, _TRACE, _TRACE_STAGES = _TRACE or [], None, None
    return log


class _Stage:
    __slots__ = ("name", "launches", "nbytes", "ev0")

    def __init__(self, name: str, launches: int, nbytes: int):
        self.name, self.launches, self.nbytes = name, launches, nbytes
        self.ev0 = None

    def __enter__(self):
        if _traced(self.name):
            self.ev0 = torch.cuda.Event(enable_timing=True)
            self.ev0.record()
        return self

    def __exit__(self, *exc):
        if _TRACE is not None and self.ev0 is not None and exc[0] is None:
            ev1 = torch.cuda.Event(enable_timing=True)
            ev1.record()
            _TRACE.append((self.name, self.ev0, ev1, self.launches, self.nbytes))
        return False


def _raw_stream(dev_index: int | None = None) -> int:
    """The current stream of a device as a raw pointer (torch's private fast
    accessor when it exists: the public one builds a Stream object)."""
    idx = torch.cuda.current_device() if dev_index is None else dev_index
    fast = getattr(torch._C, "_cuda_getCurrentRawStream", None)
    return fast(idx) if fast is not None else torch.cuda.current_stream(idx).cuda_stream


def _stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(_raw_stream())


class _NoGuard:
    __slots__ = ()

    def __enter__(self):
        return None

    def __exit__(self, *exc):
        return False


_NO_GUARD = _NoGuard()


def _on(device) -> object:
    """Make ``device`` current around a library call.

    The C functions launch on the calling thread's current device and take the
    current stream of that device; tensors placed on another GPU (a model moved
    with ``.to("cuda:1")`` and no ``torch.cuda.set_device``) would otherwise be
    handed to kernels running on the wrong device.  No-op (and no driver call)
    when the device is already current."""
    idx = torch.device(device).index
    if idx is None or idx == torch.cuda.current_device():
        return _NO_GUARD
    return torch.cuda.device(idx)


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    """Scratch buffer for one launch, reused per (device, stream).

    Launches on one stream are ordered, so reuse is safe there; another
    stream gets its own buffer.
    """
    dev = torch.device(device)
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    key = (idx, _raw_stream(idx))
    buf = _WS.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=dev)
        _WS[key] = buf
    return buf


class Cells(Sequence):
    """A checked batch of same-shape, same-dtype contiguous CUDA tensors with
    its host array of device pointers, built once and reused by every launch
    that takes the batch (the per-tensor Python work, not the launches, is
    what a 64-cell call spends its host time on).

    Either a list of tensors, or one tensor whose first dimension indexes the
    cells; then the per-cell views are made only when asked for, and the
    pointers are computed from the base address."""

    __slots__ = ("_items", "_batch", "_ptrs")

    def __init__(self, items=None, ptrs=None, batch: torch.Tensor | None = None):
        self._items = None if items is None else list(items)
        self._batch = batch
        self._ptrs = ptrs

    def __len__(self) -> int:
        return int(self._batch.shape[0]) if self._batch is not None else len(self._items)

    def __getitem__(self, i):
        if self._items is None:
            if isinstance(i, int) and i == 0:
                return self._batch[0]  # shape / dtype probes: no need for every view
            self._items = list(self._batch.unbind(0))  # one call for all the views
        return self._items[i]

    def __iter__(self):
        if self._items is None:
            self._items = list(self._batch.unbind(0))
        return iter(self._items)

    @property
    def batch(self) -> torch.Tensor | None:
        """The tensor the cells are slices of, when they are."""
        return self._batch

    def ptrs(self) -> ctypes.Array:
        if self._ptrs is None:
            if self._batch is not None:
                b = self._batch
                base, step = b.data_ptr(), b.stride(0) * b.element_size()
                self._ptrs = ptr_array(base + i * step for i in range(len(self)))
            else:
                self._ptrs = ptr_array(x.data_ptr() for x in self._items)
        return self._ptrs

    def reshape(self, *shape) -> "Cells":
        """The same cells under another shape (same storage, same pointers)."""
        if self._batch is not None and self._items is None:
            return Cells(batch=self._batch.view(len(self), *shape), ptrs=self._ptrs)
        return Cells([x.view(*shape) for x in self._items], self._ptrs)


def cells(xs: Sequence[torch.Tensor], what: str = "cells") -> Cells:
    """Check a batch once; later launches on it skip the checks."""
    return _cells(xs, what)


def split(batch: torch.Tensor) -> Cells:
    """``batch[i]`` for every i, as a batch of cells (one allocation; views and
    pointers are derived from it)."""
    return Cells(batch=batch)


def _ptrs(seq) -> ctypes.Array:
    return seq.ptrs() if isinstance(seq, Cells) else ptr_array(t.data_ptr() for t in seq)


def _cells(xs: Sequence[torch.Tensor], what: str) -> Cells:
    if isinstance(xs, Cells) and 0 < len(xs) <= KVC.MAX_CELLS:
        return xs
    if isinstance(xs, Cells):
        xs = list(xs)
    xs = tuple(xs)
    if not xs:
        raise ValueError(f"{what}: empty cell batch")
    if len(xs) > KVC.MAX_CELLS:
        raise ValueError(f"{what}: at most {KVC.MAX_CELLS} cells per launch")
    x0 = xs[0]
    if not x0.is_cuda:
        raise RuntimeError(f"{what}: kvcompress_b200 runs on CUDA tensors only (got {x0.device})")
    for x in xs:
        if x.shape != x0.shape or x.dtype != x0.dtype or x.device != x0.device:
            raise ValueError(f"{what}: cells must share shape, dtype and device")
        if not x.is_contiguous():
            raise ValueError(f"{what}: cells must be contiguous")
    return Cells(xs)


def _views(batch: torch.Tensor) -> Cells:
    """Per-cell outputs as views of one allocation (one allocator call per
    launch instead of one per cell; each view is contiguous)."""
    return split(batch)


def _code(dtype: torch.dtype) -> int:
    try:
        return DTYPE_CODE[dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {dtype}") from None


def gram(cells: Sequence[torch.Tensor], omega: torch.Tensor | None) -> torch.Tensor:
    """``[A^T A | A^T Omega | sum(A*A)]`` per cell, A = cell viewed (rows, p)."""
    cells = _cells(cells, "gram")
    p = cells[0].shape[-1]
    rows = cells[0].numel() // p
    k = 0 if omega is None else int(omega.shape[1])
    if omega is not None:
        if omega.dtype != torch.float32 or not omega.is_contiguous() or omega.shape[0] != rows:
            raise ValueError("gram: omega must be a contiguous float32 (rows, k) tensor")
    dev = cells[0].device
    out = torch.empty(len(cells), p * p + p * k + 1, dtype=torch.float64, device=dev)
    L = lib()
    ws_n = L.kvc_gram_workspace_bytes(len(cells), rows, p, k)
    ws = workspace(ws_n, dev)
    nbytes = len(cells) * cells[0].numel() * cells[0].element_size() + (0 if omega is None else omega.numel() * 4)
    with _on(dev), _Stage("gram", 3, nbytes):
        check(L.kvc_gram(len(cells), _ptrs(cells), rows, p,
                         _code(cells[0].dtype), omega.data_ptr() if omega is not None else None, k,
                         out.data_ptr(), ws.data_ptr(), ws.numel(), _stream()), "kvc_gram")
    return out


def sketch_solve(g: torch.Tensor, *, mode: int, side: int, p: int, n_other: int, k: int, rank: int,
                 n_power: int, omega: torch.Tensor | None, basis_dtype: torch.dtype,
                 gram_stride: int | None = None, want_sv2: bool = True):
    """Run the per-cell small solver; returns ``(basis, tail, sv2)``.

    ``want_sv2=False`` asks for no squared singular values (``sv2`` is then
    None): wide sketches then take the solver's complement path, whose basis
    spans the same Ritz subspace without ordering its columns."""
    n = int(g.shape[0])
    dev = g.device
    L = lib()
    if side == KVC.SIDE_LEFT:
        basis = torch.empty(n, p, rank, dtype=basis_dtype, device=dev)
    else:
        basis = torch.empty(n, p, rank, dtype=torch.float64, device=dev)
    tail = torch.empty(n, dtype=torch.float64, device=dev)
    sv2 = torch.empty(n, rank, dtype=torch.float64, device=dev) if want_sv2 else None
    kk = k if mode == KVC.SVD_RANDOMISED else 0
    ws_n = L.kvc_sketch_solve_workspace_bytes(n, mode, p, kk)
    ws = workspace(ws_n, dev)
    stride = gram_stride if gram_stride is not None else int(g.shape[1])
    with _on(dev), _Stage("sketch_solve", 1, g.numel() * 8):
        check(L.kvc_sketch_solve(n, mode, side, p, n_other, kk, rank, n_power, g.data_ptr(), stride,
                                 omega.data_ptr() if omega is not None else None, basis.data_ptr(),
                                 _code(basis.dtype), sv2.data_ptr() if sv2 is not None else None, tail.data_ptr(),
                                 ws.data_ptr(),
                                 ws.numel(), _stream()), "kvc_sketch_solve")
    return basis, tail, sv2


def project_feature(xs: Sequence[torch.Tensor], u_feature: Sequence[torch.Tensor]) -> list[torch.Tensor]:
    """``x_proj`` of each cell in token-unfolding layout ``(T, m * rd)``."""
    xs = _cells(xs, "project_feature")
    m, t, d = xs[0].shape
    rd = int(u_feature[0].shape[1])
    outs = _views(torch.empty(len(xs), t, m * rd, dtype=xs[0].dtype, device=xs[0].device))
    nbytes = len(xs) * (xs[0].numel() + outs[0].numel()) * xs[0].element_size()
    with _on(xs[0].device), _Stage("project_feature", 1, nbytes):
        check(lib().kvc_project_feature(len(xs), _ptrs(xs), m, t, d,
                                        _code(xs[0].dtype), _ptrs(u_feature),
                                        rd, _ptrs(outs), _stream()),
              "kvc_project_feature")
    return outs


def apply_basis(a: Sequence[torch.Tensor], mat: torch.Tensor) -> list[torch.Tensor]:
    """``U = A M`` per cell; ``mat`` is (n_cells, p, r) float64."""
    a = _cells(a, "apply_basis")
    rows, p = a[0].shape
    r = int(mat.shape[2])
    outs = _views(torch.empty(len(a), rows, r, dtype=a[0].dtype, device=a[0].device))
    nbytes = len(a) * (a[0].numel() + outs[0].numel()) * a[0].element_size()
    with _on(a[0].device), _Stage("apply_basis", 1, nbytes):
        check(lib().kvc_apply_basis(len(a), _ptrs(a), rows, p,
                                    _code(a[0].dtype), mat.data_ptr(), r,
                                    _ptrs(outs), _stream()), "kvc_apply_basis")
    return outs


def core(x_proj_t: Sequence[torch.Tensor], u_token: Sequence[torch.Tensor], m: int, rd: int) -> list[torch.Tensor]:
    """Tucker core ``(m, rt, rd)`` per cell (tucker.py:261)."""
    x_proj_t = _cells(x_proj_t, "core")
    t = int(x_proj_t[0].shape[0])
    rt = int(u_token[0].shape[1])
    dev = x_proj_t[0].device
    outs = _views(torch.empty(len(x_proj_t), m, rt, rd, dtype=x_proj_t[0].dtype, device=dev))
    L = lib()
    ws_n = L.kvc_core_workspace_bytes(len(outs), t, m, rd, rt)
    ws = workspace(ws_n, dev)
    nbytes = len(outs) * (x_proj_t[0].numel() + u_token[0].numel()) * x_proj_t[0].element_size()
    with _on(dev), _Stage("core", 2, nbytes):
        check(L.kvc_core(len(outs), _ptrs(x_proj_t),
                         _ptrs(u_token), t, m, rd, rt,
                         _code(x_proj_t[0].dtype), _ptrs(outs), ws.data_ptr(),
                         ws.numel(), _stream()), "kvc_core")
    return outs


def _factor_ptrs(factors, n):
    if factors is None:
        z = ptr_array([0] * n)
        return z, z, z, 0, 0
    core_, ut, ud = factors
    return (_ptrs(core_), _ptrs(ut),
            _ptrs(ud), int(ut[0].shape[1]), int(ud[0].shape[1]))


def residual_stats(xs, factors, proj, *, bits: int, symmetric: bool, scale_mode: int,
                   stat_dtype: torch.dtype):
    """Scale / zero point of the (rotated) residual of each cell."""
    xs = _cells(xs, "residual_stats")
    m, t, d = xs[0].shape
    dev = xs[0].device
    n = len(xs)
    ns = d if scale_mode == KVC.SCALE_CHANNEL else 1
    shape = (d,) if scale_mode == KVC.SCALE_CHANNEL else ()
    scales = _views(torch.empty((n,) + shape, dtype=torch.float32, device=dev))
    zps = _views(torch.empty((n,) + shape, dtype=torch.int32, device=dev))
    del ns
    cp, up, dp, rt, rd = _factor_ptrs(factors, n)
    L = lib()
    ws_n = L.kvc_residual_stats_workspace_bytes(n, m * t, d, rd)
    ws = workspace(ws_n, dev)
    with _on(dev), _Stage("residual_stats", 2, n * xs[0].numel() * xs[0].element_size()):
        check(L.kvc_residual_stats(n, _ptrs(xs), m, t, d, _code(xs[0].dtype),
                                   cp, up, dp, rt, rd, proj.data_ptr() if proj is not None else None,
                                   bits, int(symmetric), scale_mode, _code(stat_dtype),
                                   _ptrs(scales),
                                   _ptrs(zps), ws.data_ptr(), ws.numel(),
                                   _stream()), "kvc_residual_stats")
    return scales, zps


def residual_quant(xs, factors, proj, scales, zps, *, bits: int, symmetric: bool, scale_mode: int,
                   group_size: int | None, stat_dtype: torch.dtype, arith_dtype: torch.dtype):
    """Quantised, bit-packed residual codes ``(m*T, ceil(d*bits/8))`` per cell.

    With ``scale_mode == SCALE_GROUP`` the per-row group scales are computed
    here: pass ``scales = zps = None`` and receive them back.
    """
    xs = _cells(xs, "residual_quant")
    m, t, d = xs[0].shape
    dev = xs[0].device
    n = len(xs)
    if scale_mode == KVC.SCALE_GROUP:
        ng = d // int(group_size)
        scales = _views(torch.empty(n, m * t, ng, dtype=torch.float32, device=dev))
        zps = _views(torch.empty(n, m * t, ng, dtype=torch.int32, device=dev))
    cb = (d * bits + 7) // 8
    codes = _views(torch.empty(n, m * t, cb, dtype=torch.uint8, device=dev))
    cp, up, dp, rt, rd = _factor_ptrs(factors, n)
    ws = workspace(lib().kvc_residual_quant_workspace_bytes(n, m * t, d, rd), dev)
    nbytes = n * (xs[0].numel() * xs[0].element_size() + codes[0].numel())
    with _on(dev), _Stage("residual_quant", 1, nbytes):
        check(lib().kvc_residual_quant(n, _ptrs(xs), m, t, d,
                                       _code(xs[0].dtype), cp, up, dp, rt, rd,
                                       proj.data_ptr() if proj is not None else None, bits,
                                       int(symmetric), scale_mode, int(group_size or 0),
                                       _code(stat_dtype), _code(arith_dtype),
                                       _ptrs(scales),
                                       _ptrs(zps),
                                       _ptrs(codes), ws.data_ptr(), ws.numel(),
                                       _stream()),
              "kvc_residual_quant")
    return codes, scales, zps


def decompress(shape, out_dtype: torch.dtype, *, codes=None, scales=None, zps=None, bits: int = 0,
               symmetric: bool = True, scale_mode: int = KVC.SCALE_CHANNEL, group_size=None,
               factors=None, proj=None, t0: int = 0, t1: int | None = None, n_cells: int = 1,
               device=None, out=None):
    """Fused decode of ``n_cells`` cells; returns a list of ``(m, t1-t0, d)``."""
    m, t, d = (int(s) for s in shape)
    t1 = t if t1 is None else int(t1)
    if out is None:
        out = _views(torch.empty(n_cells, m, t1 - t0, d, dtype=out_dtype, device=device))
    n = len(out)
    cp, up, dp, rt, rd = _factor_ptrs(factors, n)
    fdt = _code(factors[0][0].dtype) if factors is not None else KVC.F16
    if bits > 0:
        c_arr = _ptrs(codes)
        s_arr = _ptrs(scales)
        z_arr = _ptrs(zps)
    else:
        c_arr = s_arr = z_arr = ptr_array([0] * n)
    dev0 = out[0].device
    ws = workspace(lib().kvc_decompress_workspace_bytes(n, m * t, d, rd), dev0)
    nbytes = n * out[0].numel() * out[0].element_size()
    if bits > 0:
        nbytes += sum(c.numel() for c in codes) * (t1 - t0) // t
    with _on(dev0), _Stage("decompress", 1, nbytes):
        check(lib().kvc_decompress(n, c_arr, s_arr, z_arr, bits, int(symmetric), scale_mode,
                                   int(group_size or 0), cp, up, dp, fdt, m, t, d, rt, rd,
                                   proj.data_ptr() if proj is not None else None, t0, t1,
                                   _code(out_dtype), _ptrs(out),
                                   ws.data_ptr(), ws.numel(), _stream()),
              "kvc_decompress")
    return out


def compress(xs, *, rt: int, rd: int, mode_f: int, k_f: int, omega_f: torch.Tensor | None, mode_t: int, k_t: int,
             omega_t: torch.Tensor | None, n_power: int, proj: torch.Tensor | None, bits: int, symmetric: bool,
             scale_mode: int, group_size: int | None, factor_dtype: torch.dtype | None,
             stat_dtype: torch.dtype = torch.float32, arith_dtype: torch.dtype = torch.float32) -> dict:
    """The whole compress of same-shape cells in one C call (``kvc_compress``).

    Returns batches (first dimension = cell): ``core`` (n, m, rt, rd),
    ``u_token`` (n, T, rt), ``u_feature`` (n, d, rd) in the cell dtype, the
    same in ``factor_dtype`` under ``*_stored`` (None when the dtypes agree),
    ``tail_token`` / ``tail_feature`` (n,) float64 and, with ``bits > 0``,
    ``scale`` / ``zero_point`` / ``codes``."""
    xs = _cells(xs, "compress")
    with _on(xs[0].device):
        return _compress(xs, rt=rt, rd=rd, mode_f=mode_f, k_f=k_f, omega_f=omega_f, mode_t=mode_t, k_t=k_t,
                         omega_t=omega_t, n_power=n_power, proj=proj, bits=bits, symmetric=symmetric,
                         scale_mode=scale_mode, group_size=group_size, factor_dtype=factor_dtype,
                         stat_dtype=stat_dtype, arith_dtype=arith_dtype)


def _compress(xs, *, rt, rd, mode_f, k_f, omega_f, mode_t, k_t, omega_t, n_power, proj, bits, symmetric,
              scale_mode, group_size, factor_dtype, stat_dtype, arith_dtype) -> dict:
    m, t, d = (int(v) for v in xs[0].shape)
    dev, dt = xs[0].device, xs[0].dtype
    n = len(xs)
    L = lib()
    core_ = torch.empty(n, m, rt, rd, dtype=dt, device=dev)
    ut = torch.empty(n, t, rt, dtype=dt, device=dev)
    ud = torch.empty(n, d, rd, dtype=dt, device=dev)
    cast = factor_dtype is not None and factor_dtype != dt
    core_f = torch.empty(n, m, rt, rd, dtype=factor_dtype, device=dev) if cast else None
    ut_f = torch.empty(n, t, rt, dtype=factor_dtype, device=dev) if cast else None
    ud_f = torch.empty(n, d, rd, dtype=factor_dtype, device=dev) if cast else None
    tails = (torch.empty(n, dtype=torch.float64, device=dev), torch.empty(n, dtype=torch.float64, device=dev))
    # the tails also land in pinned host memory as soon as the solves finish;
    # ``tails_ready`` is recorded then (the caller can read them while the
    # residual passes run)
    tails_host = torch.empty(2 * n, dtype=torch.float64, pin_memory=True)
    tails_ready = torch.cuda.Event()
    tails_ready.record()  # creates the CUDA event the library records again
    out = {"core": core_, "u_token": ut, "u_feature": ud, "core_stored": core_f, "u_token_stored": ut_f,
           "u_feature_stored": ud_f, "tail_token": tails[0], "tail_feature": tails[1],
           "tails_host": tails_host, "tails_ready": tails_ready,
           "scale": None, "zero_point": None, "codes": None}
    sc = zp = codes = None
    if bits > 0:
        if scale_mode == KVC.SCALE_CHANNEL:
            sshape = (n, d)
        elif scale_mode == KVC.SCALE_GROUP:
            sshape = (n, m * t, d // int(group_size))
        else:
            sshape = (n,)
        sc = torch.empty(sshape, dtype=torch.float32, device=dev)
        zp = torch.empty(sshape, dtype=torch.int32, device=dev)
        codes = torch.empty(n, m * t, (d * bits + 7) // 8, dtype=torch.uint8, device=dev)
        out.update(scale=sc, zero_point=zp, codes=codes)
    ws = workspace(L.kvc_compress_workspace_bytes(n, m, t, d, _code(dt), rt, rd, mode_f, k_f, mode_t, k_t, bits,
                                                  scale_mode), dev)
    ptr = lambda x: x.data_ptr() if x is not None else None  # noqa: E731
    evs = None
    if _TRACE is not None:
        evs = [torch.cuda.Event(enable_timing=True) if _traced(name) else None
               for name, _ in _COMPRESS_STAGES for _ in range(2)]
        for e in evs:
            if e is not None:
                e.record()  # creates the CUDA event the library records again
        # stages without events get null pointers, which the library skips
        ev_arr = ptr_array(e.cuda_event if e is not None else 0 for e in evs)  # kept by the library until reset
        check(L.kvc_trace_stages(ev_arr, len(evs)), "kvc_trace_stages")
    try:
        check(L.kvc_compress(n, _ptrs(xs), m, t, d, _code(dt), rt, rd, mode_f, k_f, ptr(omega_f), mode_t, k_t,
                             ptr(omega_t), n_power, ptr(proj), bits, int(symmetric), scale_mode, int(group_size or 0),
                             _code(stat_dtype), _code(arith_dtype), _code(factor_dtype or dt), ptr(core_), ptr(ut),
                             ptr(ud), ptr(core_f), ptr(ut_f), ptr(ud_f), ptr(tails[0]), ptr(tails[1]),
                             tails_host.data_ptr(), tails_ready.cuda_event, ptr(sc),
                             ptr(zp), ptr(codes), ws.data_ptr(), ws.numel(), _stream()), "kvc_compress")
    finally:
        if evs is not None:
            L.kvc_trace_stages(None, 0)
            del ev_arr
    if evs is not None:
        x_bytes = n * xs[0].numel() * xs[0].element_size()
        xp_bytes = n * t * m * rd * xs[0].element_size()
        sizes = {"gram": x_bytes, "sketch_solve": 0, "project_feature": x_bytes + xp_bytes, "apply_basis": xp_bytes,
                 "core": xp_bytes, "residual_stats": x_bytes,
                 "residual_quant": x_bytes + (codes.numel() if codes is not None else 0), "cast": 0}
        for i, (name, launches) in enumerate(_COMPRESS_STAGES):
            if (name in ("residual_stats", "residual_quant") and bits == 0) or evs[2 * i] is None:
                continue
            nb = xp_bytes if (name == "gram" and i > 0) else sizes[name]
            _TRACE.append((name, evs[2 * i], evs[2 * i + 1], launches, nb))
    return out


# kvc_compress's stages in order, with the kernels each launches on the
# tensor-core path (the stage timing of the bench)
_COMPRESS_STAGES = [("gram", 4), ("sketch_solve", 1), ("project_feature", 1), ("gram", 3), ("sketch_solve", 1),
                    ("apply_basis", 1), ("core", 2), ("residual_stats", 4), ("residual_quant", 2), ("cast", 3)]


class DecodePlan:
    """A tensor-core decode prepared once for token-range runs
    (``kvc_decode_plan_init`` / ``kvc_decode_plan_run``).

    Holds the plan's host bytes, its own device workspace (the cells' B
    images and the Tucker row terms) and references to the payload tensors,
    which must not change while the plan lives.  ``run(t0, t1)`` decodes
    tokens ``[t0, t1)`` of every cell with one or two kernel launches, bit for bit
    the rows ``decompress`` gives for that range.  Use one plan from one
    stream at a time.  ``DecodePlan.make`` returns None for layouts without a
    tensor-core plan (decode those with ``decompress``).
    """

    def __init__(self, L, buf, ws, keep, shape, out_dtype, n, device, m, t, d, bits):
        self._L, self._buf, self._ws, self._keep = L, buf, ws, keep
        self.shape, self.out_dtype, self.n_cells, self.device = shape, out_dtype, n, device
        self._m, self._t, self._d, self._bits = m, t, d, bits
        self._codes_bytes = [c.numel() for c in keep[0]] if bits > 0 else [0] * n

    @classmethod
    def make(cls, shape, out_dtype: torch.dtype, *, codes, scales, zps, bits: int, symmetric: bool = True,
             scale_mode: int = KVC.SCALE_CHANNEL, group_size=None, factors=None, proj=None):
        m, t, d = (int(s) for s in shape)
        n = len(codes)
        L = lib()
        cp, up, dp, rt, rd = _factor_ptrs(factors, n)
        fdt = _code(factors[0][0].dtype) if factors is not None else KVC.F16
        dev = codes[0].device
        ws = torch.empty(max(int(L.kvc_decompress_workspace_bytes(n, m * t, d, rd)), 256), dtype=torch.uint8,
                         device=dev)
        nb = int(L.kvc_decode_plan_bytes())
        buf = ctypes.create_string_buffer(nb)
        with _on(dev):
            rc = L.kvc_decode_plan_init(buf, nb, n, _ptrs(codes), _ptrs(scales), _ptrs(zps), bits, int(symmetric),
                                        scale_mode, int(group_size or 0), cp, up, dp, fdt, m, t, d, rt, rd,
                                        proj.data_ptr() if proj is not None else None, _code(out_dtype),
                                        ws.data_ptr(), ws.numel(), _stream())
        if rc == KVC.ERR_UNSUPPORTED:
            return None
        check(rc, "kvc_decode_plan_init")
        keep = (list(codes), list(scales), list(zps), factors, proj)
        return cls(L, buf, ws, keep, (m, t, d), out_dtype, n, dev, m, t, d, bits)

    def run(self, t0: int, t1: int, out=None) -> Cells:
        m, t, d = self._m, self._t, self._d
        if out is None:
            out = _views(torch.empty(self.n_cells, m, t1 - t0, d, dtype=self.out_dtype, device=self.device))
        nbytes = self.n_cells * out[0].numel() * out[0].element_size() + sum(self._codes_bytes) * (t1 - t0) // t
        with _on(self.device), _Stage("decode_range", 2, nbytes):
            check(self._L.kvc_decode_plan_run(self._buf, len(self._buf), int(t0), int(t1), _ptrs(out), _stream()),
                  "kvc_decode_plan_run")
        return out


def decompress_noalloc(shape, out_dtype: torch.dtype, *, codes=None, scales=None, zps=None, bits: int = 0,
                       symmetric: bool = True, scale_mode: int = KVC.SCALE_CHANNEL, group_size=None,
                       factors=None, proj=None, t0: int = 0, t1: int | None = None, out=None):
    """``decompress`` through ``kvc_decompress_noalloc``: no workspace.

    For callers that must not allocate device scratch: the library decodes
    in its own fixed per-device array (``KVC.NOALLOC_SCRATCH_BYTES``) and
    rejects larger decodes.  ``out`` must be given (this function allocates
    nothing on the device).  Calls that overlap on the device race on that
    array; calls on one stream are ordered.
    """
    if out is None:
        raise ValueError("decompress_noalloc: pass preallocated `out` tensors")
    m, t, d = (int(s) for s in shape)
    t1 = t if t1 is None else int(t1)
    n = len(out)
    cp, up, dp, rt, rd = _factor_ptrs(factors, n)
    fdt = _code(factors[0][0].dtype) if factors is not None else KVC.F16
    if bits > 0:
        c_arr = _ptrs(codes)
        s_arr = _ptrs(scales)
        z_arr = _ptrs(zps)
    else:
        c_arr = s_arr = z_arr = ptr_array([0] * n)
    with _on(out[0].device):  # the stream, the library's scratch and the tensors on one device
        check(lib().kvc_decompress_noalloc(n, c_arr, s_arr, z_arr, bits, int(symmetric), scale_mode,
                                           int(group_size or 0), cp, up, dp, fdt, m, t, d, rt, rd,
                                           proj.data_ptr() if proj is not None else None, t0, t1,
                                           _code(out_dtype), _ptrs(out), _stream()),
              "kvc_decompress_noalloc")
    return out


def set_kernel_policy(policy: int) -> None:
    """0: tensor-core kernels where eligible (default); 1: SIMT kernels only;
    2: as 0 with the stats pass in its fp16 mode too; 3: bf16 operands with
    the row-major quantise pass; 4: bf16 operands with the feature-major
    quantise pass."""
    check(lib().kvc_set_kernel_policy(int(policy)), "kvc_set_kernel_policy")


def launch_count() -> int:
    """Kernels this host thread has launched through the library so far."""
    return int(lib().kvc_launch_count())


def device_error() -> int:
    """Read and clear the device error word (synchronises the device)."""
    code = ctypes.c_int(0)
    check(lib().kvc_device_error(ctypes.byref(code)), "kvc_device_error")
    return int(code.value)


def cast(x: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """``x.to(dtype)`` through the extension (fp32/fp16/bf16/float8_e4m3fn)."""
    if not x.is_cuda:
        raise RuntimeError("cast: CUDA tensors only")
    x = x.contiguous()
    out = torch.empty(x.shape, dtype=dtype, device=x.device)
    with _on(x.device), _Stage("cast", 1, x.numel() * (x.element_size() + out.element_size())):
        check(lib().kvc_cast(x.numel(), x.data_ptr(), _code(x.dtype), out.data_ptr(), _code(dtype),
                             _stream()), "kvc_cast")
    return out
