"""ctypes binding of the C ABI (``include/relm_mp.h``, ``librelm_mp_b200.so``).

This is the binding a non-torch host (or a test) uses: plain device pointers,
sizes, a caller-allocated workspace and a CUDA stream. The helpers at the
bottom take torch CUDA tensors for convenience, allocate outputs and the
workspace with torch, and call the C entry points on the current stream.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "librelm_mp_b200.so"

FLOAT32, FLOAT64, BFLOAT16, FLOAT16 = 0, 1, 2, 3
MODE_SUM, MODE_LOGSUMEXP, MODE_LOGSUMEXP_BACKWARD = 0, 1, 2
MODE_MEAN = 2  # LGAN ops
STATUS_NAMES = {
    0: "RELM_MP_OK",
    1: "RELM_MP_ERR_INVALID_ARGUMENT",
    2: "RELM_MP_ERR_INDEX_OUT_OF_RANGE",
    3: "RELM_MP_ERR_WORKSPACE_TOO_SMALL",
    4: "RELM_MP_ERR_UNSUPPORTED",
    5: "RELM_MP_ERR_CUDA",
}

# Every symbol the header declares, with (restype, argtypes).
_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_SZ = ctypes.c_size_t
_INT = ctypes.c_int
_STR = ctypes.c_char_p


class Plan(ctypes.Structure):
    _fields_ = [
        ("num_edges", ctypes.c_int64),
        ("num_rows", ctypes.c_int64),
        ("gather_rows", ctypes.c_int64),
        ("num_tiles", ctypes.c_int64),
        ("tile_items", ctypes.c_int32),
        ("flags", ctypes.c_uint32),
        ("row_ptr", ctypes.c_void_p),
        ("gidx", ctypes.c_void_p),
        ("tile_row", ctypes.c_void_p),
        ("tile_edge", ctypes.c_void_p),
        ("device_flags", ctypes.c_void_p),
    ]


_PLANP = ctypes.POINTER(Plan)


class LganGraph(ctypes.Structure):
    """relm_mp_lgan_graph: the RR / TN / NN edge lists of the LGAN ops."""

    _fields_ = [
        ("rr_src", ctypes.c_void_p),
        ("rr_dst", ctypes.c_void_p),
        ("num_rr", ctypes.c_int64),
        ("tn_rel", ctypes.c_void_p),
        ("tn_ent", ctypes.c_void_p),
        ("num_tn", ctypes.c_int64),
        ("nn_rel", ctypes.c_void_p),
        ("nn_ent", ctypes.c_void_p),
        ("num_nn", ctypes.c_int64),
        ("relation_count", ctypes.c_int64),
        ("entity_dim_size", ctypes.c_int64),
    ]


_GRAPHP = ctypes.POINTER(LganGraph)


class LseForm(ctypes.Structure):
    """relm_mp_lse_form: the smoothed logsumexp's beta and eps."""

    _fields_ = [("beta", ctypes.c_double), ("eps", ctypes.c_double)]


_FORMP = ctypes.POINTER(LseForm)

SIGNATURES: dict[str, tuple] = {
    "relm_mp_status_string": (_STR, [_INT]),
    "relm_mp_build_info": (_STR, []),
    "relm_mp_last_error": (_STR, []),
    "relm_mp_kernel_launches": (ctypes.c_ulonglong, []),
    "relm_mp_fanout_scatter_workspace_bytes": (_SZ, [_I64, _I64, _I64, _I64, _INT]),
    "relm_mp_fanout_scatter": (_INT, [_INT, _P, _I64, _I64, _P, _P, _I64, _I64, _P, _P, _SZ, _P]),
    "relm_mp_fanout_scatter_backward_workspace_bytes": (_SZ, [_I64, _I64, _I64, _INT]),
    "relm_mp_fanout_scatter_backward": (_INT, [_INT, _P, _I64, _I64, _P, _P, _I64, _I64, _P, _P, _SZ, _P]),
    "relm_mp_fanin_reduce_workspace_bytes": (_SZ, [_I64, _I64, _I64, _INT, _INT]),
    "relm_mp_fanin_reduce": (_INT, [_INT, _P, _I64, _I64, _P, _P, _I64, _I64, _INT, _P, _P, _SZ, _P]),
    "relm_mp_fanin_reduce_sum_backward_workspace_bytes": (_SZ, [_I64, _I64, _I64, _INT]),
    "relm_mp_fanin_reduce_sum_backward": (_INT, [_INT, _P, _I64, _I64, _P, _P, _I64, _I64, _P, _P, _SZ, _P]),
    "relm_mp_fanin_reduce_logsumexp_backward_workspace_bytes": (_SZ, [_I64, _I64, _I64, _INT]),
    "relm_mp_fanin_reduce_logsumexp_backward": (
        _INT,
        [_INT, _P, _P, _I64, _P, _I64, _I64, _P, _P, _I64, _I64, _P, _P, _SZ, _P],
    ),
    "relm_mp_fanin_reduce_noalloc": (_INT, [_INT, _P, _I64, _I64, _P, _P, _I64, _I64, _INT, _P, _P]),
    "relm_mp_plan_bytes": (_SZ, [_I64, _I64]),
    "relm_mp_plan_scratch_bytes": (_SZ, [_I64, _I64]),
    "relm_mp_plan_build": (_INT, [_P, _P, _I64, _I64, _I64, _STR, _STR, _P, _SZ, _P, _SZ, _P, _PLANP]),
    "relm_mp_plan_build_ex": (
        _INT,
        [_P, _P, _I64, _I64, _I64, _I64, _STR, _STR, _INT, _P, _SZ, _P, _SZ, _P, _PLANP],
    ),
    "relm_mp_plan_stats_bytes": (_SZ, []),
    "relm_mp_plan_build_identity": (_INT, [_P, _I64, _I64, _I64, _P, _SZ, _P, _PLANP]),
    "relm_mp_plan_build_trusted": (_INT, [_P, _P, _I64, _I64, _I64, _P, _SZ, _P, _SZ, _P, _PLANP]),
    "relm_mp_plan_build_start": (_INT, [_P, _P, _I64, _I64, _I64, _I64, _P, _SZ, _P, _SZ, _P, _P]),
    "relm_mp_plan_build_finish": (
        _INT,
        [_P, _P, _I64, _I64, _I64, _I64, _STR, _STR, _INT, _P, _SZ, _P, _SZ, _P, _P, _PLANP],
    ),
    "relm_mp_plan_reduce_scratch_bytes": (_SZ, [_PLANP, _I64, _INT, _INT]),
    "relm_mp_plan_read_flags": (_INT, [_PLANP, _P]),
    "relm_mp_plan_gather_last": (_INT, [_PLANP, _INT, _P, _I64, _P, _P]),
    "relm_mp_plan_gather_cover": (_INT, [_PLANP, _P, ctypes.POINTER(ctypes.c_int), _P]),
    "relm_mp_plan_gather_cover_scratch_bytes": (_SZ, [_PLANP]),
    "relm_mp_plan_gather_cover_ex": (
        _INT, [_PLANP, _P, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(_I64), _P, _SZ, _P]
    ),
    "relm_mp_plan_cover_scratch_bytes": (_SZ, [_I64, _I64, _I64]),
    "relm_mp_plan_build_cover": (
        _INT,
        [_P, _P, _I64, _I64, _I64, _I64, _STR, _STR, _INT, _P, _SZ, _P, _SZ, _P, ctypes.POINTER(ctypes.c_int),
         ctypes.POINTER(_I64), _P, _PLANP],
    ),
    "relm_mp_plan_nonempty_rows": (_INT, [_PLANP, ctypes.POINTER(_I64), _P]),
    "relm_mp_pack_index": (_INT, [_P, _INT, _P, _P]),
    "relm_mp_plan_scatter_logsumexp_backward": (_INT, [_PLANP, _INT, _P, _P, _P, _I64, _P, _P, _P]),
    "relm_mp_plan_scatter_rows": (_INT, [_PLANP, _INT, _P, _I64, _P, _P, _P]),
    "relm_mp_plan_reduce": (_INT, [_PLANP, _INT, _INT, _P, _I64, _P, _P, _SZ, _P]),
    "relm_mp_plan_logsumexp_backward": (_INT, [_PLANP, _INT, _P, _P, _P, _I64, _P, _P, _SZ, _P]),
    "relm_mp_plan_reduce_ex": (_INT, [_PLANP, _INT, _P, _I64, _P, _P, _INT, _P, _P, _SZ, _P]),
    "relm_mp_plan_reduce_lse": (_INT, [_PLANP, _INT, _FORMP, _P, _I64, _P, _P, _SZ, _P]),
    "relm_mp_plan_logsumexp_backward_ex": (_INT, [_PLANP, _INT, _FORMP, _P, _P, _P, _I64, _P, _P, _SZ, _P]),
    "relm_mp_plan_scatter_logsumexp_backward_ex": (_INT, [_PLANP, _INT, _FORMP, _P, _P, _P, _I64, _P, _P, _P]),
    "relm_mp_plan_scatter_rows_div": (_INT, [_PLANP, _INT, _P, _I64, _P, _P, _P, _P]),
    "relm_mp_plan_gather_counts": (_INT, [_PLANP, _P, _P]),
    "relm_mp_plan_gather_rows_div": (_INT, [_PLANP, _P, _INT, _P, _I64, _P, _P, _P]),
    "relm_mp_divide_rows": (_INT, [_INT, _P, _I64, _I64, _P, _P, _P]),
    "relm_mp_lgan_workspace_bytes": (_SZ, [_GRAPHP, _I64, _I64, _INT]),
    "relm_mp_lgan_relation_graph_step": (_INT, [_INT, _GRAPHP, _P, _I64, _INT, _P, _P, _P, _P, _SZ, _P]),
    "relm_mp_lgan_relation_graph_step_backward": (
        _INT,
        [_INT, _GRAPHP, _P, _P, _P, _I64, _INT, _P, _P, _SZ, _P],
    ),
    "relm_mp_lgan_pool_reduce": (
        _INT,
        [_INT, _GRAPHP, _P, _I64, _I64, _P, _P, _INT, _P, _P, _P, _P, _SZ, _P],
    ),
    "relm_mp_lgan_pool_reduce_backward": (
        _INT,
        [_INT, _GRAPHP, _P, _P, _P, _I64, _I64, _P, _P, _INT, _P, _P, _SZ, _P],
    ),
}

_LIB: ctypes.CDLL | None = None


class IndexPart(ctypes.Structure):
    """relm_mp_index_part: out[start + i] = src[i] * mul + add."""

    _fields_ = [("src", ctypes.c_void_p), ("len", ctypes.c_int64), ("mul", ctypes.c_int64), ("add", ctypes.c_int64)]


def pack_index(parts, muls, adds, out=None):
    """Concatenate index tensors `parts` (int64, one CUDA device) as
    part * mul + add, in one launch per 64 parts."""

    torch = _torch()
    parts = [p.contiguous() for p in parts]
    total = sum(int(p.numel()) for p in parts)
    device = parts[0].device
    if out is None:
        out = torch.empty(total, dtype=torch.int64, device=device)
    arr = (IndexPart * max(len(parts), 1))()
    for i, (p, m, a) in enumerate(zip(parts, muls, adds)):
        arr[i] = IndexPart(_ptr(p), int(p.numel()), int(m), int(a))
    check(lib().relm_mp_pack_index(ctypes.cast(arr, ctypes.c_void_p), len(parts), _ptr(out), _stream(device)))
    return out


class RelmMpError(RuntimeError):
    def __init__(self, status: int, message: str):
        self.status = status
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")


def lib() -> ctypes.CDLL:
    """Load the library (RTLD_GLOBAL not needed) and declare every signature."""

    global _LIB
    if _LIB is None:
        if not LIB_PATH.is_file():
            raise FileNotFoundError(f"{LIB_PATH} missing: build it with `python -m relmo_b200.build`.")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = handle
    return _LIB


def check(status: int) -> None:
    if status != 0:
        raise RelmMpError(status, lib().relm_mp_last_error().decode())


# ---- torch helpers -----------------------------------------------------------------


def _torch():
    import torch

    return torch


def dtype_code(t) -> int:
    torch = _torch()
    codes = {torch.float32: FLOAT32, torch.float64: FLOAT64, torch.bfloat16: BFLOAT16, torch.float16: FLOAT16}
    if t.dtype not in codes:
        raise TypeError(f"unsupported dtype {t.dtype}")
    return codes[t.dtype]


def _ptr(t) -> int | None:
    return t.data_ptr() if t is not None and t.numel() > 0 else None


def _stream(device) -> int:
    return _torch().cuda.current_stream(device).cuda_stream


def _workspace(nbytes: int, device):
    return _torch().empty(max(int(nbytes), 1), dtype=_torch().uint8, device=device)


def divide_rows(x, counts, out=None):
    """out[r] = x[r] / max(counts[r], 1) (relm_mp_divide_rows; out may be x)."""

    x = x.contiguous()
    if out is None:
        out = _torch().empty_like(x)
    check(lib().relm_mp_divide_rows(dtype_code(x), _ptr(x), x.size(0), x.size(1), _ptr(counts.contiguous()),
                                    _ptr(out), _stream(x.device)))
    return out


def fanout_scatter(x, src, flat_dst, out_rows: int, out=None):
    torch = _torch()
    x, src, flat_dst = x.contiguous(), src.contiguous(), flat_dst.contiguous()
    emb = x.size(1)
    if out is None:
        out = torch.empty((int(out_rows), emb), dtype=x.dtype, device=x.device)
    ws = _workspace(
        lib().relm_mp_fanout_scatter_workspace_bytes(src.numel(), x.size(0), int(out_rows), emb, dtype_code(x)), x.device
    )
    check(lib().relm_mp_fanout_scatter(
        dtype_code(x), _ptr(x), x.size(0), emb, _ptr(src), _ptr(flat_dst), src.numel(), int(out_rows),
        _ptr(out), ws.data_ptr(), ws.numel(), _stream(x.device),
    ))
    return out


def fanout_scatter_backward(grad_out, src, flat_dst, x_rows: int):
    torch = _torch()
    g, src, flat_dst = grad_out.contiguous(), src.contiguous(), flat_dst.contiguous()
    emb = g.size(1)
    out = torch.empty((int(x_rows), emb), dtype=g.dtype, device=g.device)
    ws = _workspace(
        lib().relm_mp_fanout_scatter_backward_workspace_bytes(src.numel(), int(x_rows), emb, dtype_code(g)), g.device
    )
    check(lib().relm_mp_fanout_scatter_backward(
        dtype_code(g), _ptr(g), g.size(0), emb, _ptr(src), _ptr(flat_dst), src.numel(), int(x_rows),
        _ptr(out), ws.data_ptr(), ws.numel(), _stream(g.device),
    ))
    return out


def fanin_reduce(rel, flat_src, dst, dim_size: int, mode: int):
    torch = _torch()
    rel, flat_src, dst = rel.contiguous(), flat_src.contiguous(), dst.contiguous()
    emb = rel.size(1)
    out = torch.empty((int(dim_size), emb), dtype=rel.dtype, device=rel.device)
    ws = _workspace(
        lib().relm_mp_fanin_reduce_workspace_bytes(flat_src.numel(), int(dim_size), emb, dtype_code(rel), int(mode)),
        rel.device,
    )
    check(lib().relm_mp_fanin_reduce(
        dtype_code(rel), _ptr(rel), rel.size(0), emb, _ptr(flat_src), _ptr(dst), flat_src.numel(), int(dim_size),
        int(mode), _ptr(out), ws.data_ptr(), ws.numel(), _stream(rel.device),
    ))
    return out


def fanin_reduce_sum_backward(grad_out, flat_src, dst, rel_rows: int):
    torch = _torch()
    g, flat_src, dst = grad_out.contiguous(), flat_src.contiguous(), dst.contiguous()
    emb = g.size(1)
    out = torch.empty((int(rel_rows), emb), dtype=g.dtype, device=g.device)
    ws = _workspace(
        lib().relm_mp_fanin_reduce_sum_backward_workspace_bytes(flat_src.numel(), int(rel_rows), emb, dtype_code(g)),
        g.device,
    )
    check(lib().relm_mp_fanin_reduce_sum_backward(
        dtype_code(g), _ptr(g), g.size(0), emb, _ptr(flat_src), _ptr(dst), flat_src.numel(), int(rel_rows),
        _ptr(out), ws.data_ptr(), ws.numel(), _stream(g.device),
    ))
    return out


def fanin_reduce_logsumexp_backward(grad_out, rel, flat_src, dst, lse_out, rel_rows: int):
    torch = _torch()
    g, rel, o = grad_out.contiguous(), rel.contiguous(), lse_out.contiguous()
    flat_src, dst = flat_src.contiguous(), dst.contiguous()
    emb = g.size(1)
    out = torch.empty((int(rel_rows), emb), dtype=g.dtype, device=g.device)
    ws = _workspace(
        lib().relm_mp_fanin_reduce_logsumexp_backward_workspace_bytes(flat_src.numel(), int(rel_rows), emb, dtype_code(g)),
        g.device,
    )
    check(lib().relm_mp_fanin_reduce_logsumexp_backward(
        dtype_code(g), _ptr(g), _ptr(rel), rel.size(0), _ptr(o), o.size(0), emb, _ptr(flat_src), _ptr(dst),
        flat_src.numel(), int(rel_rows), _ptr(out), ws.data_ptr(), ws.numel(), _stream(g.device),
    ))
    return out


NOALLOC_SCRATCH_BYTES = 16 << 20


def fanin_reduce_noalloc(rel, flat_src, dst, dim_size: int, mode: int, out=None):
    """fanin_reduce through the entry point that takes its scratch from the
    library's static device array (no workspace argument)."""

    torch = _torch()
    rel, flat_src, dst = rel.contiguous(), flat_src.contiguous(), dst.contiguous()
    emb = rel.size(1)
    if out is None:
        out = torch.empty((int(dim_size), emb), dtype=rel.dtype, device=rel.device)
    check(lib().relm_mp_fanin_reduce_noalloc(
        dtype_code(rel), _ptr(rel), rel.size(0), emb, _ptr(flat_src), _ptr(dst), flat_src.numel(), int(dim_size),
        int(mode), _ptr(out), _stream(rel.device),
    ))
    return out


class PlanHandle:
    """A plan built through the C ABI, owning its device memory (torch)."""

    def __init__(self, out_index, gather_index, num_rows: int, gather_rows: int, with_cover: bool = False):
        """gather_index None: the identity (edge e gathers row e). with_cover:
        build through relm_mp_plan_build_cover (self.cover, self.repeats)."""

        torch = _torch()
        out_index = out_index.contiguous()
        gather_index = gather_index.contiguous() if gather_index is not None else None
        e = out_index.numel()
        self.memory = _workspace(lib().relm_mp_plan_bytes(e, int(num_rows)), out_index.device)
        self.plan = Plan()
        self.device = out_index.device
        if with_cover:
            scratch = _workspace(lib().relm_mp_plan_cover_scratch_bytes(e, int(num_rows), int(gather_rows)),
                                 out_index.device)
            self.cover = torch.empty(max(1, (int(gather_rows) + 31) // 32), dtype=torch.int32,
                                     device=out_index.device)
            rep = ctypes.c_int(-1)
            covered = ctypes.c_int64(-1)
            check(lib().relm_mp_plan_build_cover(
                _ptr(out_index), _ptr(gather_index), e, int(num_rows), int(num_rows), int(gather_rows), None, None,
                0, self.memory.data_ptr(), self.memory.numel(), scratch.data_ptr(), scratch.numel(), _ptr(self.cover),
                ctypes.byref(rep), ctypes.byref(covered), _stream(out_index.device), ctypes.byref(self.plan),
            ))
            self.repeats = bool(rep.value)
            self.covered = int(covered.value)
            return
        scratch = _workspace(lib().relm_mp_plan_scratch_bytes(e, int(num_rows)), out_index.device)
        check(lib().relm_mp_plan_build(
            _ptr(out_index), _ptr(gather_index), e, int(num_rows), int(gather_rows), None, None,
            self.memory.data_ptr(), self.memory.numel(), scratch.data_ptr(), scratch.numel(),
            _stream(out_index.device), ctypes.byref(self.plan),
        ))

    def read_flags(self) -> int:
        """Copies the plan's device flags into plan.flags (later planned calls
        launch only the kernels the plan needs); returns plan.flags."""

        check(lib().relm_mp_plan_read_flags(ctypes.byref(self.plan), _stream(self.device)))
        return int(self.plan.flags)

    def row_ptr(self):
        """row_ptr of the plan as a CPU int64 tensor."""

        return _device_int32(self.plan.row_ptr, self.plan.num_rows + 1, self.device).cpu().long()

    def gidx(self):
        """Gathered row of each edge in output-row order, as a CPU int64 tensor."""

        return _device_int32(self.plan.gidx, self.plan.num_edges, self.device).cpu().long()

    def reduce(self, table, mode: int):
        torch = _torch()
        table = table.contiguous()
        emb = table.size(1)
        out = torch.empty((self.plan.num_rows, emb), dtype=table.dtype, device=table.device)
        scratch = _workspace(
            lib().relm_mp_plan_reduce_scratch_bytes(ctypes.byref(self.plan), emb, dtype_code(table), int(mode)),
            table.device,
        )
        check(lib().relm_mp_plan_reduce(
            ctypes.byref(self.plan), dtype_code(table), int(mode), _ptr(table), emb, _ptr(out),
            scratch.data_ptr(), scratch.numel(), _stream(table.device),
        ))
        return out

    def reduce_lse(self, table, beta: float | None = None, eps: float = 0.0):
        """Logsumexp over each row's gathered rows: plain (beta None) or the
        smoothed form (relm_mp_plan_reduce_lse)."""

        torch = _torch()
        table = table.contiguous()
        emb = table.size(1)
        out = torch.empty((self.plan.num_rows, emb), dtype=table.dtype, device=table.device)
        form = ctypes.byref(LseForm(float(beta), float(eps))) if beta is not None else None
        scratch = _workspace(
            lib().relm_mp_plan_reduce_scratch_bytes(ctypes.byref(self.plan), emb, dtype_code(table), MODE_LOGSUMEXP),
            table.device,
        )
        check(lib().relm_mp_plan_reduce_lse(
            ctypes.byref(self.plan), dtype_code(table), form, _ptr(table), emb, _ptr(out),
            scratch.data_ptr(), scratch.numel(), _stream(table.device),
        ))
        return out

    def logsumexp_backward(self, grad_out, lse_out, rel, beta: float | None = None):
        """grad_rel[r] = sum over r's edges of grad_out[g] * exp(beta (rel[r] - lse_out[g]))
        (relm_mp_plan_logsumexp_backward_ex; beta None: 1)."""

        torch = _torch()
        grad_out, lse_out, rel = grad_out.contiguous(), lse_out.contiguous(), rel.contiguous()
        emb = grad_out.size(1)
        out = torch.empty((self.plan.num_rows, emb), dtype=grad_out.dtype, device=grad_out.device)
        form = ctypes.byref(LseForm(float(beta), 0.0)) if beta is not None else None
        scratch = _workspace(
            lib().relm_mp_plan_reduce_scratch_bytes(ctypes.byref(self.plan), emb, dtype_code(grad_out), 2),
            grad_out.device,
        )
        check(lib().relm_mp_plan_logsumexp_backward_ex(
            ctypes.byref(self.plan), dtype_code(grad_out), form, _ptr(grad_out), _ptr(lse_out), _ptr(rel), emb,
            _ptr(out), scratch.data_ptr(), scratch.numel(), _stream(grad_out.device),
        ))
        return out

    def reduce_ex(self, table, base=None, row_div=None, divide_by_count: bool = False, out=None):
        """out[r] = base[r] + sum / max(d_r, 1) (relm_mp_plan_reduce_ex); out may be base."""

        torch = _torch()
        table = table.contiguous()
        emb = table.size(1)
        if out is None:
            out = torch.empty((self.plan.num_rows, emb), dtype=table.dtype, device=table.device)
        scratch = _workspace(
            lib().relm_mp_plan_reduce_scratch_bytes(ctypes.byref(self.plan), emb, dtype_code(table), MODE_SUM),
            table.device,
        )
        check(lib().relm_mp_plan_reduce_ex(
            ctypes.byref(self.plan), dtype_code(table), _ptr(table), emb, _ptr(base), _ptr(row_div),
            int(bool(divide_by_count)), _ptr(out), scratch.data_ptr(), scratch.numel(), _stream(table.device),
        ))
        return out

    def gather_counts(self):
        """Edges per gathered row (int32 CUDA tensor)."""

        torch = _torch()
        counts = torch.empty(max(int(self.plan.gather_rows), 1), dtype=torch.int32, device=self.device)
        check(lib().relm_mp_plan_gather_counts(ctypes.byref(self.plan), _ptr(counts), _stream(self.device)))
        return counts[: int(self.plan.gather_rows)]

    def scatter_rows_div(self, table, row_div, cover=None):
        """out[gidx[e]] = table[row of e] / max(row_div[row], 1); cover None: every out row is an edge target."""

        torch = _torch()
        table = table.contiguous()
        emb = table.size(1)
        out = torch.empty((self.plan.gather_rows, emb), dtype=table.dtype, device=table.device)
        check(lib().relm_mp_plan_scatter_rows_div(
            ctypes.byref(self.plan), dtype_code(table), _ptr(table), emb, _ptr(row_div), _ptr(cover), _ptr(out),
            _stream(table.device),
        ))
        return out

    def gather_rows_div(self, out_index, table, row_div):
        """out[s] = table[out_index[s]] / max(row_div[out_index[s]], 1) (identity-gather plan of out_index)."""

        torch = _torch()
        table = table.contiguous()
        emb = table.size(1)
        out = torch.empty((self.plan.num_edges, emb), dtype=table.dtype, device=table.device)
        check(lib().relm_mp_plan_gather_rows_div(
            ctypes.byref(self.plan), _ptr(out_index.contiguous()), dtype_code(table), _ptr(table), emb,
            _ptr(row_div), _ptr(out), _stream(table.device),
        ))
        return out

    def gather_last(self, table):
        torch = _torch()
        table = table.contiguous()
        emb = table.size(1)
        out = torch.empty((self.plan.num_rows, emb), dtype=table.dtype, device=table.device)
        check(lib().relm_mp_plan_gather_last(
            ctypes.byref(self.plan), dtype_code(table), _ptr(table), emb, _ptr(out), _stream(table.device)
        ))
        return out


    def gather_cover(self):
        """Coverage bitmap of the gather rows (int32 device tensor of 32-row
        words) and whether any gather row is used more than once."""

        torch = _torch()
        words = max((int(self.plan.gather_rows) + 31) // 32, 1)
        cover = torch.empty(words, dtype=torch.int32, device=self.device)  # bitmap, 32 rows per word
        dups = ctypes.c_int(0)
        check(lib().relm_mp_plan_gather_cover(ctypes.byref(self.plan), _ptr(cover), ctypes.byref(dups),
                                              _stream(self.device)))
        return cover, bool(dups.value)

    def gather_cover_ex(self):
        """relm_mp_plan_gather_cover_ex (byte marks, caller scratch): (bitmap, has_dups)."""

        torch = _torch()
        words = max(1, (int(self.plan.gather_rows) + 31) // 32)
        cover = torch.empty(words, dtype=torch.int32, device=self.device)
        scratch = _workspace(lib().relm_mp_plan_gather_cover_scratch_bytes(ctypes.byref(self.plan)), self.device)
        dups = ctypes.c_int(0)
        covered = ctypes.c_int64(-1)
        check(lib().relm_mp_plan_gather_cover_ex(
            ctypes.byref(self.plan), _ptr(cover), ctypes.byref(dups), ctypes.byref(covered), scratch.data_ptr(),
            scratch.numel(), _stream(self.device),
        ))
        self.covered = int(covered.value)
        return cover, bool(dups.value)

    def nonempty_rows(self) -> int:
        rows = ctypes.c_int64(0)
        check(lib().relm_mp_plan_nonempty_rows(ctypes.byref(self.plan), ctypes.byref(rows), _stream(self.device)))
        return int(rows.value)

    def scatter_rows(self, table, cover):
        """out[gidx[e]] = table[row of e] for every edge, zeros for uncovered gather rows."""

        torch = _torch()
        table = table.contiguous()
        emb = table.size(1)
        out = torch.empty((self.plan.gather_rows, emb), dtype=table.dtype, device=table.device)
        check(lib().relm_mp_plan_scatter_rows(
            ctypes.byref(self.plan), dtype_code(table), _ptr(table), emb, _ptr(cover), _ptr(out), _stream(table.device)
        ))
        return out


# ---- LGAN ops (op-level entry points) --------------------------------------------


def _lgan_graph(rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent, relation_count: int, entity_dim_size: int):
    ix = [i.contiguous().long() for i in (rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent)]
    g = LganGraph(
        _ptr(ix[0]), _ptr(ix[1]), ix[0].numel(), _ptr(ix[2]), _ptr(ix[3]), ix[2].numel(),
        _ptr(ix[4]), _ptr(ix[5]), ix[4].numel(), int(relation_count), int(entity_dim_size),
    )
    return g, ix


def _lgan_ws(g, num_slots: int, like):
    return _workspace(lib().relm_mp_lgan_workspace_bytes(ctypes.byref(g), int(num_slots), like.size(1),
                                                         dtype_code(like)), like.device)


def lgan_relation_graph_step(x, rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent, entity_dim_size: int, mode: int):
    torch = _torch()
    x = x.contiguous()
    g, keep = _lgan_graph(rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent, x.size(0), entity_dim_size)
    x1 = torch.empty_like(x)
    tn = torch.empty((int(entity_dim_size), x.size(1)), dtype=x.dtype, device=x.device)
    nn = torch.empty_like(tn)
    ws = _lgan_ws(g, 0, x)
    check(lib().relm_mp_lgan_relation_graph_step(
        dtype_code(x), ctypes.byref(g), _ptr(x), x.size(1), int(mode), _ptr(x1), _ptr(tn), _ptr(nn),
        ws.data_ptr(), ws.numel(), _stream(x.device),
    ))
    del keep
    return x1, tn, nn


def lgan_relation_graph_step_backward(gx, gtn, gnn, rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent,
                                      relation_count: int, mode: int):
    torch = _torch()
    gx, gtn, gnn = gx.contiguous(), gtn.contiguous(), gnn.contiguous()
    g, keep = _lgan_graph(rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent, relation_count, gtn.size(0))
    out = torch.empty((int(relation_count), gx.size(1)), dtype=gx.dtype, device=gx.device)
    ws = _lgan_ws(g, 0, gx)
    check(lib().relm_mp_lgan_relation_graph_step_backward(
        dtype_code(gx), ctypes.byref(g), _ptr(gx), _ptr(gtn), _ptr(gnn), gx.size(1), int(mode), _ptr(out),
        ws.data_ptr(), ws.numel(), _stream(gx.device),
    ))
    del keep
    return out


def lgan_pool_reduce(slots, slot_to_rel, arities, rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent,
                     entity_dim_size: int, mode: int):
    torch = _torch()
    slots, s2r, ar = slots.contiguous(), slot_to_rel.contiguous().long(), arities.contiguous()
    R = ar.numel()
    g, keep = _lgan_graph(rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent, R, entity_dim_size)
    x1 = torch.empty((R, slots.size(1)), dtype=slots.dtype, device=slots.device)
    tn = torch.empty((int(entity_dim_size), slots.size(1)), dtype=slots.dtype, device=slots.device)
    nn = torch.empty_like(tn)
    ws = _lgan_ws(g, slots.size(0), slots)
    check(lib().relm_mp_lgan_pool_reduce(
        dtype_code(slots), ctypes.byref(g), _ptr(slots), slots.size(0), slots.size(1), _ptr(s2r), _ptr(ar),
        int(mode), _ptr(x1), _ptr(tn), _ptr(nn), ws.data_ptr(), ws.numel(), _stream(slots.device),
    ))
    del keep
    return x1, tn, nn


def lgan_pool_reduce_backward(gx, gtn, gnn, slot_to_rel, arities, rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent,
                              relation_count: int, mode: int):
    torch = _torch()
    gx, gtn, gnn = gx.contiguous(), gtn.contiguous(), gnn.contiguous()
    s2r, ar = slot_to_rel.contiguous().long(), arities.contiguous()
    g, keep = _lgan_graph(rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent, relation_count, gtn.size(0))
    out = torch.empty((s2r.numel(), gx.size(1)), dtype=gx.dtype, device=gx.device)
    ws = _lgan_ws(g, s2r.numel(), gx)
    check(lib().relm_mp_lgan_pool_reduce_backward(
        dtype_code(gx), ctypes.byref(g), _ptr(gx), _ptr(gtn), _ptr(gnn), gx.size(1), s2r.numel(), _ptr(s2r),
        _ptr(ar), int(mode), _ptr(out), ws.data_ptr(), ws.numel(), _stream(gx.device),
    ))
    del keep
    return out


class _DeviceArray:
    def __init__(self, ptr: int, n: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (int(n),), "typestr": typestr, "data": (int(ptr), False), "version": 3}


def _device_int32(ptr: int, n: int, device):
    """A torch view of `n` int32 values at device address `ptr` (no copy)."""

    torch = _torch()
    torch.cuda.current_stream(device).synchronize()
    if n == 0:
        return torch.empty(0, dtype=torch.int32, device=device)
    return torch.as_tensor(_DeviceArray(ptr, n, "<i4"), device=device)
