"""Python surface of the B200 runtime: contexts, plans and the hot-path ops.

Every op takes and returns torch CUDA tensors (torch is the device-memory and
stream plumbing here) and calls straight into libgnnc_b200.so through the C
ABI; nothing in this module computes on the host. 2-D feature tensors may be
row-padded views (stride(1) == 1, stride(0) >= width): the padding keeps every
row 16-byte aligned so the kernels can use vector loads.
"""

from __future__ import annotations

import ctypes
import threading
from dataclasses import dataclass

import torch

from gnnc.b200 import _lib
from gnnc.b200._lib import ACT_ELU, ACT_NONE, ACT_RELU, BF16, F32, GnncError, raise_for

__all__ = [
    "ACT_ELU",
    "ACT_NONE",
    "ACT_RELU",
    "DeviceRows",
    "Context",
    "GnncError",
    "Plan",
    "csr_from_coo",
    "empty_rows",
    "gat_aggregate",
    "gat_aggregate_noalloc",
    "gcn_aggregate",
    "gather_rows",
    "gcn_norm",
    "mean_norm",
    "peer_close",
    "peer_copy",
    "peer_export",
    "peer_open",
    "proj",
    "sage_aggregate",
    "softmax_aggregate",
    "validate_csr",
]

_DTYPES = {torch.float32: F32, torch.bfloat16: BF16}


@dataclass(frozen=True)
class DeviceRows:
    """Rows of a 2-D row-major array at a raw device address that is valid on
    `device` but not owned by torch (e.g. another process's buffer mapped by
    peer_open). Usable as the x operand of proj."""

    ptr: int
    rows: int
    cols: int
    ld: int  # row stride in elements
    dtype: torch.dtype
    device: torch.device

    def __getitem__(self, rows: slice) -> DeviceRows:
        a, b, step = rows.indices(self.rows)
        if step != 1:
            raise ValueError("DeviceRows takes contiguous row slices only")
        b = max(a, b)
        esz = torch.empty((), dtype=self.dtype).element_size()
        return DeviceRows(self.ptr + a * self.ld * esz, b - a, self.cols, self.ld, self.dtype,
                          self.device)


def _dt(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {t.dtype}; expected float32 or bfloat16") from None


def _p(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _ld(t: torch.Tensor) -> int:
    """Row stride of a 2-D feature tensor; its storage must cover every padded row."""
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError("feature tensors must be 2-D with unit column stride")
    ld = t.stride(0) if t.size(0) > 1 else max(t.stride(0), t.size(1))
    need = (t.storage_offset() + t.size(0) * ld) * t.element_size()
    if t.numel() and t.untyped_storage().nbytes() < need:
        raise ValueError("row-padded tensor whose storage does not cover the last row's padding")
    return ld


def _check_edges(plan: "Plan", *arrays: torch.Tensor | None) -> None:
    for a in arrays:
        if a is not None and a.size(0) < plan.num_edges:
            raise ValueError(f"edge array has {a.size(0)} entries, the CSR needs {plan.num_edges}")


def _check_cuda(*ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("B200 ops take CUDA tensors")


def row_stride(width: int, dtype: torch.dtype) -> int:
    """Row stride (elements) that keeps rows 16-byte aligned."""
    per = 16 // torch.empty((), dtype=dtype).element_size()
    return (width + per - 1) // per * per


def empty_rows(n: int, width: int, dtype: torch.dtype, device) -> torch.Tensor:
    """[n, width] view of an [n, row_stride(width)] buffer (16-byte aligned rows)."""
    ld = row_stride(width, dtype)
    buf = torch.empty((n, ld), dtype=dtype, device=device)
    return buf[:, :width]


class Context:
    """One libgnnc_b200 context per CUDA device per process."""

    _lock = threading.Lock()
    _by_device: dict[int, Context] = {}

    def __init__(self, device: int) -> None:
        lib = _lib.load()
        handle = ctypes.c_void_p()
        st = lib.gnnc_init(device, ctypes.byref(handle))
        if st != _lib.OK:
            raise_for(st, None, f"gnnc_init(device={device})")
        self.lib = lib
        self.handle = handle.value
        self.device = device

    @classmethod
    def get(cls, device: torch.device | int | None = None) -> Context:
        if device is None:
            idx = torch.cuda.current_device()
        elif isinstance(device, int):
            idx = device
        else:
            device = torch.device(device)
            idx = device.index if device.index is not None else torch.cuda.current_device()
        with cls._lock:
            ctx = cls._by_device.get(idx)
            if ctx is None:
                ctx = cls._by_device[idx] = Context(idx)
        return ctx

    def use_current_stream(self) -> None:
        stream = torch.cuda.current_stream(self.device).cuda_stream
        self.lib.gnnc_stream_set(self.handle, stream)

    def call(self, name: str, *args) -> None:
        self.use_current_stream()
        st = getattr(self.lib, name)(self.handle, *args)
        raise_for(st, self.handle, name)

    def synchronize(self) -> None:
        raise_for(self.lib.gnnc_synchronize(self.handle), self.handle, "gnnc_synchronize")

    def workspace_bind(self, buf: torch.Tensor | None) -> None:
        ptr = None if buf is None else buf.data_ptr()
        n = 0 if buf is None else buf.numel() * buf.element_size()
        raise_for(self.lib.gnnc_workspace_bind(self.handle, ptr, n), self.handle, "workspace_bind")


class Plan:
    """Degree-skew row schedule of one CSR (gnnc_plan_create)."""

    def __init__(
        self,
        rowptr: torch.Tensor,
        *,
        cta_threshold: int = 0,
        split_threshold: int = 0,
        ctx: Context | None = None,
    ) -> None:
        _check_cuda(rowptr)
        if rowptr.dtype != torch.int32 or not rowptr.is_contiguous():
            raise ValueError("rowptr must be a contiguous int32 CUDA tensor")
        self.ctx = ctx or Context.get(rowptr.device)
        self.n_rows = rowptr.numel() - 1
        handle = ctypes.c_void_p()
        self.ctx.use_current_stream()
        st = self.ctx.lib.gnnc_plan_create(
            self.ctx.handle,
            rowptr.data_ptr(),
            self.n_rows,
            cta_threshold,
            split_threshold,
            ctypes.byref(handle),
        )
        raise_for(st, self.ctx.handle, "gnnc_plan_create")
        self.handle = handle.value
        # rowptr is host-validated by plan creation; keep its edge span for size checks
        ends = rowptr[[0, -1]].tolist()
        self.num_edges = int(ends[1])
        self.first_edge = int(ends[0])

    def info(self) -> dict[str, int]:
        arr = (ctypes.c_int64 * 6)()
        raise_for(self.ctx.lib.gnnc_plan_info(self.handle, arr), None, "gnnc_plan_info")
        keys = ("n_rows", "n_warp_rows", "n_cta_rows", "n_split_rows", "n_segments", "max_degree")
        return dict(zip(keys, list(arr), strict=True))

    def workspace_bytes(self, width: int) -> int:
        out = ctypes.c_size_t()
        st = self.ctx.lib.gnnc_workspace_query(self.ctx.handle, self.handle, width, ctypes.byref(out))
        raise_for(st, self.ctx.handle, "gnnc_workspace_query")
        return out.value

    def __del__(self) -> None:
        h = getattr(self, "handle", None)
        if h:
            try:
                self.ctx.lib.gnnc_plan_destroy(h)
            except Exception:  # pragma: no cover - interpreter teardown
                pass
            self.handle = None


# ---------------------------------------------------------------------------
# Graph preparation
# ---------------------------------------------------------------------------


def csr_from_coo(
    edge_index: torch.Tensor, num_nodes: int, *, self_loops: bool, dedupe: bool
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor | None]:
    """COO edge_index [2,E] (int64, CUDA) -> CSR by destination.

    Returns (rowptr int32 [N+1], col int32 [E'], mult int32 [E'] or None).
    Column order within a row is ascending source id (torch coalesce order).
    """
    _check_cuda(edge_index)
    if edge_index.dim() != 2 or edge_index.size(0) != 2:
        raise ValueError("edge_index must be [2, E]")
    ei = edge_index.to(torch.int64)
    src = ei[0].contiguous()
    dst = ei[1].contiguous()
    E = src.numel()
    cap = E + (num_nodes if self_loops else 0)
    dev = edge_index.device
    rowptr = torch.empty(num_nodes + 1, dtype=torch.int32, device=dev)
    col = torch.empty(max(cap, 1), dtype=torch.int32, device=dev)
    mult = torch.empty(max(cap, 1), dtype=torch.int32, device=dev) if dedupe else None
    ctx = Context.get(dev)
    e_out = ctypes.c_int64()
    ctx.call(
        "gnnc_csr_from_coo",
        src.data_ptr(),
        dst.data_ptr(),
        E,
        num_nodes,
        int(self_loops),
        int(dedupe),
        rowptr.data_ptr(),
        col.data_ptr(),
        _p(mult),
        cap,
        ctypes.byref(e_out),
    )
    n = e_out.value
    return rowptr, col[:n], (mult[:n] if mult is not None else None)


def gcn_norm(
    rowptr: torch.Tensor, col: torch.Tensor, mult: torch.Tensor | None = None
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """PyG gcn_norm weights on a CSR that already holds its self-loops.

    Returns (deg fp32 [N], dinv fp32 [N], w fp32 [E])."""
    _check_cuda(rowptr, col, mult)
    N = rowptr.numel() - 1
    dev = rowptr.device
    deg = torch.empty(N, dtype=torch.float32, device=dev)
    dinv = torch.empty(N, dtype=torch.float32, device=dev)
    w = torch.empty(max(col.numel(), 1), dtype=torch.float32, device=dev)
    Context.get(dev).call(
        "gnnc_gcn_norm", rowptr.data_ptr(), col.data_ptr(), _p(mult), N, deg.data_ptr(),
        dinv.data_ptr(), w.data_ptr(),
    )
    return deg, dinv, w[: col.numel()]


def validate_csr(rowptr: torch.Tensor, col: torch.Tensor, n_src: int) -> None:
    """Raises GnncInvalidArgument unless the CSR indexes [0, n_src) consistently."""
    _check_cuda(rowptr, col)
    Context.get(rowptr.device).call(
        "gnnc_csr_validate", rowptr.data_ptr(), col.data_ptr(), rowptr.numel() - 1, col.numel(),
        n_src,
    )


# ---------------------------------------------------------------------------
# Projection
# ---------------------------------------------------------------------------


def proj(
    x: torch.Tensor,
    weight: torch.Tensor,
    *,
    att_src: torch.Tensor | None = None,
    att_dst: torch.Tensor | None = None,
    heads: int = 1,
    out_dtype: torch.dtype | None = None,
    out: torch.Tensor | None = None,
    asrc_out: torch.Tensor | None = None,
    adst_out: torch.Tensor | None = None,
):
    """h = x . weight^T (+ GAT attention coefficients).

    x [N,K] (fp32 or bf16, padded rows allowed; a tensor or DeviceRows);
    weight [F,K] same dtype.
    Returns h [N,F] (row-padded) or (h, asrc [N,H], adst [N,H]) when att_* given.
    out / asrc_out / adst_out: optional destination tensors (e.g. this rank's
    slot of an all-gather buffer).
    """
    if isinstance(x, DeviceRows):
        if x.device != weight.device:
            raise ValueError("x is mapped on another device than weight")
        _check_cuda(weight, att_src, att_dst)
        x_ptr, ldx, N, K = x.ptr, x.ld, x.rows, x.cols
        if x.ld < x.cols or (x.ld * torch.empty((), dtype=x.dtype).element_size()) % 16:
            raise ValueError("DeviceRows rows must be 16-byte aligned and ld >= cols")
    else:
        _check_cuda(x, weight, att_src, att_dst)
        N, K = x.shape
        x_ptr, ldx = x.data_ptr(), _ld(x)
    if x.dtype != weight.dtype:
        raise ValueError("x and weight must share a dtype")
    F = weight.size(0)
    if weight.size(1) != K:
        raise ValueError(f"weight is {tuple(weight.shape)}, x has {K} columns")
    out_dtype = out_dtype or x.dtype
    h = _out(N, F, out_dtype, x.device, out)
    att = att_src is not None
    asrc = adst = None
    if att:
        asrc = asrc_out if asrc_out is not None else torch.empty((N, heads), dtype=torch.float32, device=x.device)
        adst = adst_out if adst_out is not None else torch.empty((N, heads), dtype=torch.float32, device=x.device)
        if asrc.shape != (N, heads) or adst.shape != (N, heads) or not (asrc.is_contiguous() and adst.is_contiguous()):
            raise ValueError("asrc_out / adst_out must be contiguous [N, heads] fp32")
        att_src = att_src.reshape(-1).to(torch.float32).contiguous()
        att_dst = att_dst.reshape(-1).to(torch.float32).contiguous()
    Context.get(x.device).call(
        "gnnc_proj",
        x_ptr, _dt(x), ldx, weight.data_ptr(), _ld(weight), N, K, F,
        _p(att_src), _p(att_dst), heads, h.data_ptr(), _dt(h), _ld(h), _p(asrc), _p(adst),
    )
    return (h, asrc, adst) if att else h


# ---------------------------------------------------------------------------
# Aggregation
# ---------------------------------------------------------------------------


def _out(n: int, width: int, dtype: torch.dtype, device, out: torch.Tensor | None):
    if out is None:
        return empty_rows(n, width, dtype, device)
    if tuple(out.shape) != (n, width) or out.dtype != dtype:
        raise ValueError(f"out must be [{n},{width}] {dtype}")
    return out


def gcn_aggregate(
    plan: Plan,
    rowptr: torch.Tensor,
    col: torch.Tensor,
    w: torch.Tensor,
    h: torch.Tensor,
    *,
    bias: torch.Tensor | None = None,
    act: int = ACT_NONE,
    log_softmax: bool = False,
    out_dtype: torch.dtype = torch.float32,
    out: torch.Tensor | None = None,
    n_src: int | None = None,
) -> torch.Tensor:
    """out = A . h (+bias, act, log_softmax); A = CSR (rowptr, col, w)."""
    _check_cuda(rowptr, col, w, h, bias)
    n_rows = rowptr.numel() - 1
    F = h.size(1)
    out = _out(n_rows, F, out_dtype, h.device, out)
    _check_edges(plan, col, w)
    bias = None if bias is None else bias.to(torch.float32).contiguous()
    plan.ctx.call(
        "gnnc_gcn_aggregate",
        plan.handle, rowptr.data_ptr(), col.data_ptr(), w.data_ptr(), h.data_ptr(), _dt(h),
        _ld(h), n_rows, h.size(0) if n_src is None else n_src, F, _p(bias), act,
        int(log_softmax), out.data_ptr(), _dt(out), _ld(out),
    )
    return out


def mean_norm(rowptr: torch.Tensor, w: torch.Tensor | None = None) -> torch.Tensor:
    """SAGE mean weights: w / max(count of nonzero w in the row, 1) (w None: unit weights)."""
    _check_cuda(rowptr, w)
    n_rows = rowptr.numel() - 1
    E = int(rowptr[-1].item()) if n_rows >= 0 else 0
    if w is not None:
        w = w.to(torch.float32).contiguous()
        if w.numel() < E:
            raise ValueError(f"w has {w.numel()} entries, the CSR needs {E}")
    out = torch.empty(max(E, w.numel() if w is not None else 0), dtype=torch.float32,
                      device=rowptr.device)
    Context.get(rowptr.device).call("gnnc_mean_norm", rowptr.data_ptr(), n_rows, _p(w),
                                    out.data_ptr())
    return out


def sage_aggregate(
    plan: Plan,
    rowptr: torch.Tensor,
    col: torch.Tensor,
    w: torch.Tensor,
    h: torch.Tensor,
    root: torch.Tensor,
    *,
    bias: torch.Tensor | None = None,
    act: int = ACT_NONE,
    log_softmax: bool = False,
    out_dtype: torch.dtype = torch.float32,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """SAGEConv after its projections: out = A_mean . h + root (+bias, act, log_softmax).

    w: mean_norm weights of the CSR; root: [n_rows, F] (x . W_r^T of the rows)."""
    _check_cuda(rowptr, col, w, h, root, bias)
    n_rows = rowptr.numel() - 1
    F = h.size(1)
    if root.dim() != 2 or root.size(0) != n_rows or root.size(1) != F:
        raise ValueError(f"root must be [{n_rows}, {F}]")
    out = _out(n_rows, F, out_dtype, h.device, out)
    _check_edges(plan, col, w)
    bias = None if bias is None else bias.to(torch.float32).contiguous()
    plan.ctx.call(
        "gnnc_sage_aggregate",
        plan.handle, rowptr.data_ptr(), col.data_ptr(), w.data_ptr(), h.data_ptr(), _dt(h),
        _ld(h), root.data_ptr(), _dt(root), _ld(root), n_rows, h.size(0), F, _p(bias), act,
        int(log_softmax), out.data_ptr(), _dt(out), _ld(out),
    )
    return out


def gat_aggregate(
    plan: Plan,
    rowptr: torch.Tensor,
    col: torch.Tensor,
    h: torch.Tensor,
    asrc: torch.Tensor,
    adst: torch.Tensor,
    *,
    heads: int,
    negative_slope: float = 0.2,
    concat: bool = True,
    bias: torch.Tensor | None = None,
    act: int = ACT_NONE,
    log_softmax: bool = False,
    out_dtype: torch.dtype = torch.float32,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Fused GATConv aggregation (SDDMM, LeakyReLU, edge softmax, SpMM, epilogue)."""
    _check_cuda(rowptr, col, h, asrc, adst, bias)
    n_rows = rowptr.numel() - 1
    F = h.size(1)
    if F % heads:
        raise ValueError("feature width not divisible by heads")
    C = F // heads
    width = F if concat else C
    out = _out(n_rows, width, out_dtype, h.device, out)
    _check_edges(plan, col)
    if asrc.shape != (h.size(0), heads) or adst.shape != (n_rows, heads):
        raise ValueError("asrc must be [n_src, heads] and adst [n_rows, heads]")
    bias = None if bias is None else bias.to(torch.float32).contiguous()
    plan.ctx.call(
        "gnnc_gat_aggregate",
        plan.handle, rowptr.data_ptr(), col.data_ptr(), h.data_ptr(), _dt(h), _ld(h),
        asrc.contiguous().data_ptr(), adst.contiguous().data_ptr(), n_rows, h.size(0), heads, C,
        float(negative_slope), int(concat), _p(bias), act, int(log_softmax), out.data_ptr(),
        _dt(out), _ld(out),
    )
    return out


def softmax_aggregate(
    plan: Plan,
    rowptr: torch.Tensor,
    col: torch.Tensor,
    scores: torch.Tensor,
    h: torch.Tensor,
    *,
    heads: int = 1,
    eps: float = 1e-16,
    concat: bool = True,
    bias: torch.Tensor | None = None,
    act: int = ACT_NONE,
    log_softmax: bool = False,
    out_dtype: torch.dtype = torch.float32,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Edge softmax of given scores [E, heads] followed by the weighted SpMM."""
    _check_cuda(rowptr, col, scores, h, bias)
    n_rows = rowptr.numel() - 1
    F = h.size(1)
    C = F // heads
    width = F if concat else C
    out = _out(n_rows, width, out_dtype, h.device, out)
    scores = scores.to(torch.float32).contiguous().view(-1, heads)
    _check_edges(plan, col, scores)
    bias = None if bias is None else bias.to(torch.float32).contiguous()
    plan.ctx.call(
        "gnnc_softmax_aggregate",
        plan.handle, rowptr.data_ptr(), col.data_ptr(), scores.data_ptr(), h.data_ptr(), _dt(h),
        _ld(h), n_rows, h.size(0), heads, C, float(eps), int(concat), _p(bias), act,
        int(log_softmax), out.data_ptr(), _dt(out), _ld(out),
    )
    return out


def gat_aggregate_noalloc(
    plan: Plan,
    rowptr: torch.Tensor,
    col: torch.Tensor,
    h: torch.Tensor,
    asrc: torch.Tensor,
    adst: torch.Tensor,
    out: torch.Tensor,
    *,
    heads: int,
    negative_slope: float = 0.2,
    concat: bool = True,
    bias: torch.Tensor | None = None,
    act: int = ACT_NONE,
    log_softmax: bool = False,
) -> torch.Tensor:
    """gat_aggregate for callers that must not allocate device memory mid-run
    (a process that reserved its memory budget up front, or a runtime that owns
    all device memory through its own pool). The library call allocates
    nothing: its scratch is a fixed 16 MiB array inside the library, shared by
    every call on the device, so calls must not overlap on the GPU. The caller
    passes every input and the output `out` (its dtype picks the output dtype)."""
    _check_cuda(rowptr, col, h, asrc, adst, bias, out)
    n_rows = rowptr.numel() - 1
    F = h.size(1)
    if F % heads:
        raise ValueError("feature width not divisible by heads")
    C = F // heads
    width = F if concat else C
    if tuple(out.shape) != (n_rows, width):
        raise ValueError(f"out must be [{n_rows},{width}]")
    _check_edges(plan, col)
    if asrc.shape != (h.size(0), heads) or adst.shape != (n_rows, heads):
        raise ValueError("asrc must be [n_src, heads] and adst [n_rows, heads]")
    if not (asrc.is_contiguous() and adst.is_contiguous()):
        raise ValueError("asrc and adst must be contiguous")
    if bias is not None and not (bias.dtype == torch.float32 and bias.is_contiguous()):
        raise ValueError("bias must be a contiguous float32 tensor")
    plan.ctx.call(
        "gnnc_gat_aggregate_noalloc",
        plan.handle, rowptr.data_ptr(), col.data_ptr(), h.data_ptr(), _dt(h), _ld(h),
        asrc.data_ptr(), adst.data_ptr(), n_rows, h.size(0), heads, C, float(negative_slope),
        int(concat), _p(bias), act, int(log_softmax), out.data_ptr(), _dt(out), _ld(out),
    )
    return out


# ---------------------------------------------------------------------------
# Peer memory (CUDA IPC)
# ---------------------------------------------------------------------------

PEER_HANDLE_BYTES = 64


def peer_export(t: torch.Tensor) -> tuple[bytes, int]:
    """(handle, offset) that lets another process map the buffer holding `t`."""
    _check_cuda(t)
    ctx = Context.get(t.device)
    handle = ctypes.create_string_buffer(PEER_HANDLE_BYTES)
    off = ctypes.c_uint64()
    st = ctx.lib.gnnc_peer_export(ctx.handle, t.data_ptr(), handle, ctypes.byref(off))
    raise_for(st, ctx.handle, "gnnc_peer_export")
    return handle.raw, off.value


def peer_open(device: torch.device | int, handle: bytes, offset: int) -> int:
    """Maps another process's exported buffer on `device`; returns its address here."""
    if len(handle) != PEER_HANDLE_BYTES:
        raise ValueError(f"peer handle must be {PEER_HANDLE_BYTES} bytes")
    ctx = Context.get(device)
    ptr = ctypes.c_void_p()
    st = ctx.lib.gnnc_peer_open(ctx.handle, handle, offset, ctypes.byref(ptr))
    raise_for(st, ctx.handle, "gnnc_peer_open")
    return ptr.value


def peer_copy(dst: torch.Tensor | DeviceRows, src: torch.Tensor | DeviceRows, nbytes: int) -> None:
    """Copies nbytes from src to dst on the current stream (either may be a
    peer mapping; a copy-engine transfer)."""
    dev = dst.device
    ptr = {}
    for name, t in (("dst", dst), ("src", src)):
        if isinstance(t, DeviceRows):
            cap = t.rows * t.ld * torch.empty((), dtype=t.dtype).element_size()
            ptr[name] = t.ptr
        else:
            _check_cuda(t)
            cap = t.untyped_storage().nbytes() - t.storage_offset() * t.element_size()
            ptr[name] = t.data_ptr()
        if nbytes > cap:
            raise ValueError(f"{name} holds {cap} bytes, {nbytes} requested")
    Context.get(dev).call("gnnc_peer_copy", ptr["dst"], ptr["src"], nbytes)


def gather_rows(src: torch.Tensor | DeviceRows, idx: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """out[i] = src[idx[i]] (whole padded rows; 16-byte aligned row strides).

    src may be a DeviceRows, e.g. another process's rows mapped by peer_open:
    the kernel then reads them over NVLink with plain loads."""
    if isinstance(src, DeviceRows):
        _check_cuda(idx, out)
        if src.device != out.device:
            raise ValueError("src rows must be addressable on out's device")
        esz = torch.empty((), dtype=src.dtype).element_size()
        src_ptr, src_ld, n_src, dtype = src.ptr, src.ld, src.rows, src.dtype
    else:
        _check_cuda(src, idx, out)
        esz = src.element_size()
        src_ptr, src_ld, n_src, dtype = src.data_ptr(), src.stride(0), src.size(0), src.dtype
    if idx.dtype != torch.int32 or not idx.is_contiguous():
        raise ValueError("idx must be a contiguous int32 tensor")
    n = idx.numel()
    if out.size(0) < n or out.dtype != dtype:
        raise ValueError("out must hold len(idx) rows of src's dtype")
    row_bytes = src_ld * esz
    if out.stride(0) * esz < row_bytes:
        raise ValueError("out rows are narrower than src rows")
    Context.get(out.device).call("gnnc_gather_rows", src_ptr, row_bytes, idx.data_ptr(), n, n_src,
                                 out.data_ptr(), out.stride(0) * esz, row_bytes)
    return out


COMM_ID_BYTES = 128


def comm_unique_id(device: torch.device | int) -> bytes:
    """A new NCCL communicator id (rank 0 makes it; the ranks share it on the host)."""
    ctx = Context.get(device)
    uid = ctypes.create_string_buffer(COMM_ID_BYTES)
    raise_for(ctx.lib.gnnc_comm_unique_id(ctx.handle, uid), ctx.handle, "gnnc_comm_unique_id")
    return uid.raw


def comm_init(device: torch.device | int, uid: bytes, rank: int, nranks: int,
              timeout_ms: int | None = None) -> None:
    """Joins communicator `uid` as `rank` of `nranks`. Waits at most timeout_ms
    (default 120 s) for every rank; past it the communicator is aborted and a
    GnncError with status ERR_TIMEOUT is raised (the context stays usable)."""
    if len(uid) != COMM_ID_BYTES:
        raise ValueError(f"communicator id must be {COMM_ID_BYTES} bytes")
    ctx = Context.get(device)
    if timeout_ms is None:
        st = ctx.lib.gnnc_comm_init(ctx.handle, uid, rank, nranks)
    else:
        st = ctx.lib.gnnc_comm_init_timeout(ctx.handle, uid, rank, nranks, int(timeout_ms))
    raise_for(st, ctx.handle, "gnnc_comm_init")


def comm_wait(device: torch.device | int, timeout_ms: int) -> None:
    """Waits at most timeout_ms for the context's stream and its collectives; a
    collective that cannot finish aborts the communicator (ERR_TIMEOUT)."""
    ctx = Context.get(device)
    raise_for(ctx.lib.gnnc_comm_wait(ctx.handle, int(timeout_ms)), ctx.handle, "gnnc_comm_wait")


def allgather(send: torch.Tensor, recv: torch.Tensor) -> torch.Tensor:
    """recv = every rank's `send`, concatenated in rank order, on the context's stream."""
    _check_cuda(send, recv)
    if not (send.is_contiguous() and recv.is_contiguous()) or send.dtype != recv.dtype:
        raise ValueError("send and recv must be contiguous tensors of one dtype")
    ctx = Context.get(send.device)
    if recv.numel() % max(1, send.numel()) != 0:
        raise ValueError("recv must hold a whole number of send buffers")
    raise_for(ctx.lib.gnnc_allgather(ctx.handle, send.data_ptr(), recv.data_ptr(), send.numel(),
                                     _dt(send)), ctx.handle, "gnnc_allgather")
    return recv


def comm_destroy(device: torch.device | int) -> None:
    ctx = Context.get(device)
    raise_for(ctx.lib.gnnc_comm_destroy(ctx.handle), ctx.handle, "gnnc_comm_destroy")


def peer_close(device: torch.device | int, ptr: int, offset: int) -> None:
    ctx = Context.get(device)
    raise_for(ctx.lib.gnnc_peer_close(ctx.handle, ptr, offset), ctx.handle, "gnnc_peer_close")
