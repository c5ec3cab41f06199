"""Thin torch-facing wrappers over the C ABI (pointers, strides, current stream).

These functions do no validation beyond what is needed to build the
descriptors; the reference-shaped public functions in ``kernels.*`` perform
the reference's checks (and raise its ``ValueError`` messages) first.
"""

from __future__ import annotations

import ctypes
import functools

import torch

from . import _lib
from ._lib import AttnOpts, AttnPlan, Tensor, check, lib

_DT = {torch.float32: _lib.KV4_F32, torch.float16: _lib.KV4_F16,
       torch.bfloat16: _lib.KV4_BF16, torch.uint8: _lib.KV4_U8}


_I64x4 = ctypes.c_int64 * 4


def desc(t: torch.Tensor, host_ok: bool = False) -> Tensor:
    """kv4_tensor for ``t`` (rank <= 4, leading dims padded with size 1).
    Compute calls take device memory only (``host_ok`` is for the host-only
    planning calls)."""
    if not host_ok and not t.is_cuda:
        raise ValueError("kvint4 kernels take CUDA tensors (no CPU path)")
    n = t.dim()
    if n == 4:  # the common case, in one constructor call
        return Tensor(t.data_ptr(), _DT[t.dtype], 0, _I64x4(*t.shape), _I64x4(*t.stride()))
    if not 1 <= n <= 4:
        raise ValueError("kvint4 tensors have 1 to 4 dims")
    shape = [1] * (4 - n) + list(t.shape)
    stride = [0] * (4 - n) + list(t.stride())
    for i in range(3 - n, -1, -1):  # padded size-1 dims get the natural stride
        stride[i] = stride[i + 1] * shape[i + 1]
    d = Tensor()
    d.data = t.data_ptr()
    d.dtype = _DT[t.dtype]
    for i in range(4):
        d.shape[i] = int(shape[i])
        d.stride[i] = int(stride[i])
    return d


def _on_device(fn):
    """Run ``fn`` with its first tensor's device current.

    The library launches on the current device (tensor maps, occupancy and
    scratch addresses are per device), so a tensor on cuda:k is handled with
    cuda:k current even when the caller's current device differs, e.g. a
    model spread over several GPUs by ``device_map``."""
    @functools.wraps(fn)
    def wrapper(t, *args, **kwargs):
        idx = t.device.index if t.is_cuda else None
        if idx is None or idx == torch.cuda.current_device():
            return fn(t, *args, **kwargs)
        with torch.cuda.device(idx):
            return fn(t, *args, **kwargs)
    return wrapper


def _stream(dev: torch.device) -> int:
    """Raw handle of the current stream of ``dev`` (no Stream object built)."""
    return torch._C._cuda_getCurrentRawStream(
        dev.index if dev.index is not None else torch.cuda.current_device())


@_on_device
def quantize_into(x: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor, group_size: int,
                  tie: int = _lib.TIE_HALF_AWAY, t_off: int = 0) -> None:
    L = lib()
    dx, dp, ds = desc(x), desc(packed), desc(scales)
    check("kv4_quantize", L.kv4_quantize(ctypes.byref(dx), ctypes.byref(dp), ctypes.byref(ds),
                                         int(t_off), int(group_size), int(tie), _stream(x.device)))


@_on_device
def append_kv(k, v, k_packed, k_scales, v_packed, v_scales, pos: int, group_size: int,
              tie: int = _lib.TIE_HALF_AWAY) -> None:
    L = lib()
    ds = [desc(t) for t in (k, v, k_packed, k_scales, v_packed, v_scales)]
    check("kv4_append_kv", L.kv4_append_kv(*[ctypes.byref(d) for d in ds], int(pos),
                                           int(group_size), int(tie), _stream(k.device)))


@_on_device
def dequantize_into(packed: torch.Tensor, scales: torch.Tensor, out: torch.Tensor,
                    group_size: int) -> None:
    L = lib()
    dp, ds, do = desc(packed), desc(scales), desc(out)
    check("kv4_dequantize", L.kv4_dequantize(ctypes.byref(dp), ctypes.byref(ds),
                                             ctypes.byref(do), int(group_size),
                                             _stream(packed.device)))


# --------------------------------------------------------------------------
# attention
# --------------------------------------------------------------------------
_WS: dict = {}
_COUNTER_RESERVE = 1 << 16  # zeroed tail of every workspace: room for 16384 units' counters


def _workspace(dev: torch.device, plan: AttnPlan) -> torch.Tensor | None:
    """Per (device, stream) scratch buffer for split-sequence partials.

    Layout: partial data from the front (never past ``numel - reserve``), a
    zero-initialised tail of ``reserve`` bytes whose end holds the kernel's
    per-unit counters.  The kernel returns the counters to zero, and no call
    writes data into the tail, so the tail stays zero between calls."""
    nbytes = int(plan.workspace_bytes)
    if nbytes <= 0:
        return None
    # unit counters plus first-level merge-group counters (8 parts per group)
    groups = (int(plan.max_parts) + 7) // 8
    counters = (int(plan.units) * 4 * (1 + (groups if groups > 1 else 0)) + 15) // 16 * 16
    data = nbytes - counters
    reserve = max(_COUNTER_RESERVE, counters)
    key = (dev.index, _stream(dev))
    buf, res = _WS.get(key, (None, 0))
    if buf is None or res < reserve or buf.numel() - res < data:
        res = max(res, reserve)
        size = max(data, 1 << 20) + res
        if buf is not None:
            size = max(size, buf.numel())
        buf = torch.zeros(size, dtype=torch.uint8, device=dev)
        _WS[key] = (buf, res)
    return buf


def _opts(force_generic=False, tiles_per_cta=0, max_ctas=0, debug_drop_last_tile=False,
          early_start=False):
    if not (force_generic or tiles_per_cta or max_ctas or debug_drop_last_tile or early_start):
        return None
    o = AttnOpts()
    o.force_generic = int(bool(force_generic))
    o.tiles_per_cta = int(tiles_per_cta)
    o.max_ctas = int(max_ctas)
    o.debug_drop_last_tile = int(bool(debug_drop_last_tile))
    o.early_start = int(bool(early_start))
    return o


_EARLY = AttnOpts()
_EARLY.early_start = 1
_EARLY_REF = ctypes.byref(_EARLY)


def plan(q, kp, ks, vp, vs, out, group_size, is_causal=False, **kw) -> AttnPlan:
    L = lib()
    ds = [desc(t, host_ok=True) for t in (q, kp, ks, vp, vs, out)]
    o = _opts(**kw)
    p = AttnPlan()
    check("kv4_attention_plan",
          L.kv4_attention_plan(*[ctypes.byref(d) for d in ds], int(group_size), int(is_causal),
                               ctypes.byref(o) if o else None, ctypes.byref(p)))
    return p


@_on_device
def attention_into(q, kp, ks, vp, vs, out, group_size: int, is_causal: bool = False,
                   sm_scale: float = 0.0, **kw) -> None:
    L = lib()
    ds = [desc(t) for t in (q, kp, ks, vp, vs, out)]
    o = _opts(**kw)
    optr = ctypes.byref(o) if o else None
    refs = [ctypes.byref(d) for d in ds]
    st = _stream(q.device)

    def call(ws, nbytes):
        return L.kv4_attention(*refs, int(group_size), int(is_causal), float(sm_scale), ws,
                               nbytes, optr, st)

    check("kv4_attention", _with_workspace(q.device, call, ds, group_size, is_causal, optr))


@_on_device
def prefill_attention_into(q, kp, ks, vp, vs, out, group_size: int, is_causal: bool = False,
                           sm_scale: float = 0.0, *, strict: bool = True) -> bool:
    """Tensor-core prefill kernel (``kv4_prefill_attention``).  Returns False
    when the shape or layout is outside what the kernel takes (only with
    ``strict=False``; otherwise that raises ``Kv4Error``)."""
    L = lib()
    refs = [ctypes.byref(desc(t)) for t in (q, kp, ks, vp, vs, out)]
    rc = L.kv4_prefill_attention(*refs, int(group_size), int(is_causal), float(sm_scale),
                                 _stream(q.device))
    if not strict and rc in (_lib.KV4_ERR_UNSUPPORTED, _lib.KV4_ERR_LAYOUT, _lib.KV4_ERR_DTYPE):
        return False
    check("kv4_prefill_attention", rc)
    return True


def _with_workspace(dev: torch.device, call, ds, group_size, is_causal, optr) -> int:
    """Run ``call(ws_ptr, ws_bytes)`` with this (device, stream)'s workspace.
    The common case plans nothing: the library reports KV4_ERR_WORKSPACE
    (before launching anything) when the buffer is too small, and then the
    plan sizes a larger one and the call is repeated."""
    buf = _WS.get((dev.index, _stream(dev)), (None, 0))[0]
    rc = call(buf.data_ptr() if buf is not None else None, buf.numel() if buf is not None else 0)
    if rc == _lib.KV4_ERR_WORKSPACE:
        L = lib()
        p = AttnPlan()
        check("kv4_attention_plan",
              L.kv4_attention_plan(*[ctypes.byref(d) for d in ds], int(group_size),
                                   int(is_causal), optr, ctypes.byref(p)))
        buf = _workspace(dev, p)
        rc = call(buf.data_ptr() if buf is not None else None,
                  buf.numel() if buf is not None else 0)
    return rc


_DESC_MEMO: dict = {}


def _desc_ref(t: torch.Tensor):
    """``byref`` of a descriptor of ``t``, memoised on (address, dtype, shape,
    strides): a decode loop passes the same activation buffers every step."""
    key = (t.data_ptr(), t.dtype, t.shape, t.stride())
    r = _DESC_MEMO.get(key)
    if r is None:
        if len(_DESC_MEMO) > 512:
            _DESC_MEMO.clear()
        d = desc(t)
        r = _DESC_MEMO[key] = (d, ctypes.byref(d))
    return r[1]


@_on_device
def append_attention_descs(q, k_new, v_new, cache_descs, out, group_size: int,
                           is_causal: bool = False, tie_mode: int = _lib.TIE_HALF_AWAY,
                           sm_scale: float = 0.0, early_start: bool = False) -> None:
    """``append_attention_into`` with prebuilt descriptors of the four cache
    views (a decode loop keeps them per layer and only updates the length).
    ``early_start``: the caller guarantees the kernel launched just before on
    the stream writes no row of these views except the previous decode row
    (``kv4_attn_opts.early_start``)."""
    L = lib()
    rq, rk, rv, ro = _desc_ref(q), _desc_ref(k_new), _desc_ref(v_new), _desc_ref(out)
    st = _stream(q.device)
    buf = _WS.get((q.device.index, st), (None, 0))[0]
    args = (rq, rk, rv, *[ctypes.byref(d) for d in cache_descs], ro, int(group_size),
            int(tie_mode), int(is_causal), float(sm_scale))
    optr = _EARLY_REF if early_start else None
    rc = L.kv4_append_attention(*args, buf.data_ptr() if buf is not None else None,
                                buf.numel() if buf is not None else 0, optr, st)
    if rc == _lib.KV4_ERR_WORKSPACE:  # first call on this stream: size the workspace
        ds = [desc(q), *cache_descs, desc(out)]

        def call(ws, nbytes):
            return L.kv4_append_attention(*args, ws, nbytes, optr, st)

        rc = _with_workspace(q.device, call, ds, group_size, is_causal, optr)
    check("kv4_append_attention", rc)


@_on_device
def append_attention_into(q, k_new, v_new, kp, ks, vp, vs, out, group_size: int,
                          is_causal: bool = False, tie_mode: int = _lib.TIE_HALF_AWAY,
                          sm_scale: float = 0.0, **kw) -> None:
    """Quantize ``k_new``/``v_new`` [B, Hkv, n, d] into the LAST n rows of the
    cache views ``kp, ks, vp, vs`` (which already span the new rows), then
    attend over all rows: one launch for n == 1 on the fast path
    (``kv4_append_attention``)."""
    L = lib()
    ds = [desc(t) for t in (q, kp, ks, vp, vs, out)]
    dn = [desc(t) for t in (k_new, v_new)]
    o = _opts(**kw)
    optr = ctypes.byref(o) if o else None
    refs = [ctypes.byref(d) for d in ds]
    st = _stream(q.device)

    def call(ws, nbytes):
        return L.kv4_append_attention(refs[0], ctypes.byref(dn[0]), ctypes.byref(dn[1]),
                                      *refs[1:], int(group_size), int(tie_mode), int(is_causal),
                                      float(sm_scale), ws, nbytes, optr, st)

    check("kv4_append_attention",
          _with_workspace(q.device, call, ds, group_size, is_causal, optr))


@_on_device
def append_kv_paged(k, v, k_pages, ks_pages, v_pages, vs_pages, slot_mapping: torch.Tensor,
                    group_size: int, tie: int = _lib.TIE_HALF_AWAY) -> None:
    """Quantize k, v [B, Hkv, n, d] into the page pools at ``slot_mapping``
    (int32 [B * n] on the device: page * page_size + row; < 0 skips)."""
    if slot_mapping.dtype != torch.int32 or not slot_mapping.is_contiguous() or \
            slot_mapping.device != k.device:
        raise ValueError("slot_mapping must be a contiguous int32 tensor on the device of k")
    L = lib()
    ds = [desc(t) for t in (k, v, k_pages, ks_pages, v_pages, vs_pages)]
    check("kv4_append_kv_paged",
          L.kv4_append_kv_paged(*[ctypes.byref(d) for d in ds], slot_mapping.data_ptr(),
                                int(group_size), int(tie), _stream(k.device)))


def paged_plan(q, k_pages, ks_pages, v_pages, vs_pages, max_blocks: int, max_seq_len: int,
               group_size: int, **kw) -> AttnPlan:
    L = lib()
    ds = [desc(t, host_ok=True) for t in (q, k_pages, ks_pages, v_pages, vs_pages)]
    o = _opts(**kw)
    p = AttnPlan()
    check("kv4_attention_paged_plan",
          L.kv4_attention_paged_plan(*[ctypes.byref(d) for d in ds], int(max_blocks),
                                     int(max_seq_len), int(group_size),
                                     ctypes.byref(o) if o else None, ctypes.byref(p)))
    return p


@_on_device
def attention_paged_into(q, k_pages, ks_pages, v_pages, vs_pages, block_table: torch.Tensor,
                         seq_lens: torch.Tensor, max_seq_len: int, out, group_size: int,
                         is_causal: bool = False, sm_scale: float = 0.0, **kw) -> None:
    """Attention over a paged INT4 cache (``kv4_attention_paged``):
    block_table int32 [B, max_blocks], seq_lens int32 [B], both on the device."""
    for t, name in ((block_table, "block_table"), (seq_lens, "seq_lens")):
        if t.dtype != torch.int32 or t.device != q.device:
            raise ValueError(f"{name} must be an int32 tensor on the device of q")
    if block_table.dim() != 2 or block_table.stride(1) != 1 or not seq_lens.is_contiguous():
        raise ValueError("block_table must be [B, max_blocks] with unit column stride")
    L = lib()
    ds = [desc(t) for t in (q, k_pages, ks_pages, v_pages, vs_pages, out)]
    p = paged_plan(q, k_pages, ks_pages, v_pages, vs_pages, block_table.shape[1], max_seq_len,
                   group_size, **kw)
    ws = _workspace(q.device, p)
    o = _opts(**kw)
    check("kv4_attention_paged",
          L.kv4_attention_paged(*[ctypes.byref(d) for d in ds[:5]], block_table.data_ptr(),
                                block_table.stride(0), block_table.shape[1], seq_lens.data_ptr(),
                                int(max_seq_len), ctypes.byref(ds[5]), int(group_size),
                                int(is_causal), float(sm_scale),
                                ws.data_ptr() if ws is not None else None,
                                ws.numel() if ws is not None else 0,
                                ctypes.byref(o) if o else None, _stream(q.device)))


@_on_device
def attention_partial_into(q, kp, ks, vp, vs, part_o, part_lse, k_offset: int, sk_total: int,
                           group_size: int, is_causal: bool = False, sm_scale: float = 0.0,
                           **kw) -> None:
    L = lib()
    ds = [desc(t) for t in (q, kp, ks, vp, vs, part_o)]
    dl = desc(part_lse.unsqueeze(-1) if part_lse.dim() == q.dim() - 1 else part_lse)
    o = _opts(**kw)
    optr = ctypes.byref(o) if o else None
    p = AttnPlan()
    check("kv4_attention_plan",
          L.kv4_attention_plan(*[ctypes.byref(d) for d in ds], int(group_size), int(is_causal),
                               optr, ctypes.byref(p)))
    ws = _workspace(q.device, p)
    check("kv4_attention_partial",
          L.kv4_attention_partial(*[ctypes.byref(d) for d in ds], ctypes.byref(dl),
                                  int(k_offset), int(sk_total), int(group_size), int(is_causal),
                                  float(sm_scale), ws.data_ptr() if ws is not None else None,
                                  ws.numel() if ws is not None else 0, optr, _stream(q.device)))


@_on_device
def lse_combine_into(parts_o: torch.Tensor, parts_lse: torch.Tensor, out: torch.Tensor) -> None:
    """parts_o f32 [P, rows, d] contiguous, parts_lse f32 [P, rows] contiguous."""
    L = lib()
    if not (parts_o.is_contiguous() and parts_lse.is_contiguous()):
        raise ValueError("parts must be contiguous")
    if parts_o.dtype != torch.float32 or parts_lse.dtype != torch.float32:
        raise ValueError("parts must be float32")
    do = desc(out)
    check("kv4_lse_combine", L.kv4_lse_combine(parts_o.data_ptr(), parts_lse.data_ptr(),
                                               int(parts_o.shape[0]), ctypes.byref(do),
                                               _stream(out.device)))


def device_error(dev: torch.device | None = None) -> int:
    """Read and clear the device error word set by bounded waits."""
    L = lib()
    flag = ctypes.c_int(0)
    dev = dev or torch.device("cuda", torch.cuda.current_device())
    check("kv4_device_error", L.kv4_device_error(_stream(dev), ctypes.byref(flag)))
    return flag.value
