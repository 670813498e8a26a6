"""Torch-facing wrappers over the libpk C ABI.

``PagedKVPool`` owns (as torch tensors) every device buffer the kernels use:
the K/V pages, the page table, the free ring, per-slot counters, the error
word and the conv time cache.  Each method checks shapes on the host, then
makes one C call on the current CUDA stream.
"""
from __future__ import annotations

import ctypes
import threading

import torch

from . import _lib
from ._lib import check, lib

DTYPES = {torch.float32: _lib.PK_DTYPE_F32, torch.bfloat16: _lib.PK_DTYPE_BF16}


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def layer_norm(x: torch.Tensor, ln, ln2=None):
    """nn.LayerNorm ``ln`` over the last dim of ``x`` (one libpk launch); with
    ``ln2`` also ``ln2(ln(x))`` from the same launch, returned as a pair.
    Widths the kernel does not take, or non-CUDA tensors, go through
    torch.nn.functional.layer_norm."""
    D = x.shape[-1]
    vec = 8 if x.dtype == torch.bfloat16 else 4
    ok = (x.is_cuda and x.dtype in DTYPES and D % (32 * vec) == 0
          and D // (32 * vec) in (1, 2, 4, 8) and ln.weight.dtype == x.dtype
          and (ln2 is None or ln2.weight.dtype == x.dtype))
    if not ok:
        y = torch.nn.functional.layer_norm(x, (D,), ln.weight, ln.bias, ln.eps)
        if ln2 is None:
            return y
        return y, torch.nn.functional.layer_norm(y, (D,), ln2.weight, ln2.bias, ln2.eps)
    x2 = x.reshape(-1, D)
    if x2.stride(-1) != 1 or x2.stride(0) % vec or x2.data_ptr() % 16:
        x2 = x2.contiguous()
    rows = x2.shape[0]
    y = torch.empty((rows, D), dtype=x.dtype, device=x.device)
    y2 = torch.empty_like(y) if ln2 is not None else None
    check(lib().pk_layer_norm(
        x2.data_ptr(), x2.stride(0), rows, D, ln.weight.data_ptr(), ln.bias.data_ptr(),
        float(ln.eps), y.data_ptr(), D,
        _ptr(ln2.weight) if ln2 is not None else None, _ptr(ln2.bias) if ln2 is not None else None,
        float(ln2.eps) if ln2 is not None else 0.0, _ptr(y2), D, DTYPES[x.dtype],
        _stream(x.device)), "pk_layer_norm")
    y = y.reshape(x.shape)
    return y if ln2 is None else (y, y2.reshape(x.shape))


GEMM_EPILOGUES = {"store": _lib.PK_GEMM_STORE, "silu": _lib.PK_GEMM_SILU,
                  "residual": _lib.PK_GEMM_RESIDUAL, "residual_relu": _lib.PK_GEMM_RESIDUAL_RELU,
                  "bias": _lib.PK_GEMM_BIAS}
_gemm_error: dict = {}


def _rows(t: torch.Tensor, width: int) -> torch.Tensor:
    """t as [rows, width] with unit column stride, 16-byte aligned rows."""
    t2 = t.reshape(-1, width)
    if t2.stride(-1) != 1 or t2.stride(0) % 8 or t2.data_ptr() % 16:
        t2 = t2.contiguous()
    return t2


def gemm_supported(a: torch.Tensor, weight: torch.Tensor) -> bool:
    """Shapes and types pk_gemm_bf16 takes: bf16 CUDA operands, K and N
    multiples of 64, the weight's rows contiguous and 16-byte aligned."""
    return (a.is_cuda and a.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16
            and weight.dim() == 2 and a.shape[-1] == weight.shape[1]
            and weight.shape[1] % 64 == 0 and weight.shape[0] % 64 == 0
            and weight.stride(1) == 1 and weight.stride(0) % 8 == 0
            and weight.data_ptr() % 16 == 0)


def gemm(a: torch.Tensor, weight: torch.Tensor, epilogue: str = "store",
         residual: torch.Tensor | None = None, alpha: float = 1.0,
         bias: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """epilogue(a @ weight.T) on the tcgen05 tensor cores (pk_gemm_bf16):
    "store" -> acc, "silu" -> acc * sigmoid(acc), "residual" -> residual +
    alpha * acc, "residual_relu" -> max(residual + alpha * acc, 0), "bias" ->
    acc + bias.  a [..., K], weight [N, K] (an nn.Linear weight), bf16;
    ``residual`` [..., N] may have strided rows; ``out`` a contiguous [M, N]."""
    K, N = weight.shape[1], weight.shape[0]
    a2 = _rows(a, K)
    M = a2.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=a.dtype, device=a.device)
    elif not out.is_contiguous() or out.numel() != M * N:
        raise ValueError("out must be a contiguous [M, N] tensor")
    r2 = None
    if epilogue in ("residual", "residual_relu"):
        r2 = _rows(residual, N)
    if epilogue == "bias" and (bias is None or not bias.is_contiguous()):
        raise ValueError("the bias epilogue needs a contiguous bias")
    err = _gemm_error.get(a.device)
    if err is None:
        err = _gemm_error[a.device] = torch.zeros(1, dtype=torch.int32, device=a.device)
    check(lib().pk_gemm_bf16(a2.data_ptr(), a2.stride(0), weight.data_ptr(), weight.stride(0), M,
                             N, K, out.data_ptr(), N, GEMM_EPILOGUES[epilogue], _ptr(r2),
                             r2.stride(0) if r2 is not None else 0, _ptr(bias), float(alpha),
                             err.data_ptr(), _stream(a.device)), "pk_gemm_bf16")
    return out.reshape(*a.shape[:-1], N)


def gemm_error_word(device) -> int:
    err = _gemm_error.get(torch.device(device))
    return 0 if err is None else int(err.item())


def pages_per_stream(left: int, chunk: int, page_size: int) -> int:
    return int(lib().pk_pages_per_stream(left, chunk, page_size))


def ring_size(left: int, chunk: int, page_size: int) -> int:
    return int(lib().pk_ring_size(left, chunk, page_size))


class PagedKVPool:
    """Paged K/V window + conv cache for ``num_slots`` stream slots.

    kv          [num_pages, L, 2, H, page_size, dh] model dtype (head-major pages)
    page_table  [num_slots, ring]                 int32, -1 = none
    free_ring   [num_pages]                       int32
    ring_ctr    [2]                               int64 head / tail
    meta        [num_slots, 8]                    int32 counters (PK_META_*)
    error       [1]                               int32 PK_DEV_* bits
    win_desc    [num_slots, 128]                  int32 this step's window descriptors
    conv        [num_slots, L, D, kernel - 1]     model dtype (ModelCache.conv layout)
    """

    def __init__(self, num_layers, dim, num_heads, att_context, num_slots, *, num_pages=None,
                 page_size=16, conv_kernel=9, dtype=torch.bfloat16, device="cuda",
                 page_order=None):
        if dtype not in DTYPES:
            raise TypeError(f"dtype {dtype} not handled (float32 or bfloat16)")
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("PagedKVPool needs a CUDA device")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.num_layers, self.dim, self.num_heads = num_layers, dim, num_heads
        self.left, right = int(att_context[0]), int(att_context[1])
        self.chunk = right + 1
        self.window = self.left + self.chunk
        self.page_size = page_size
        self.num_slots = num_slots
        self.dtype = dtype
        self.conv_kernel = conv_kernel
        self.per_stream = pages_per_stream(self.left, self.chunk, page_size)
        self.ring = ring_size(self.left, self.chunk, page_size)
        self.num_pages = int(num_pages or num_slots * self.per_stream)
        dev = self.device
        self.kv = torch.zeros((self.num_pages, num_layers, 2, num_heads, page_size, dim // num_heads),
                              dtype=dtype, device=dev)
        self.page_table = torch.full((num_slots, self.ring), -1, dtype=torch.int32, device=dev)
        self.free_ring = torch.empty(self.num_pages, dtype=torch.int32, device=dev)
        self.ring_ctr = torch.zeros(2, dtype=torch.int64, device=dev)
        self.meta = torch.zeros((num_slots, _lib.META_STRIDE), dtype=torch.int32, device=dev)
        self.error = torch.zeros(1, dtype=torch.int32, device=dev)
        self.win_desc = torch.zeros((num_slots, _lib.WIN_STRIDE), dtype=torch.int32, device=dev)
        self.conv = torch.zeros((num_slots, num_layers, dim, conv_kernel - 1), dtype=dtype, device=dev)
        d = _lib.PagedKVDesc(
            kv=self.kv.data_ptr(), page_table=self.page_table.data_ptr(),
            free_ring=self.free_ring.data_ptr(), ring_ctr=self.ring_ctr.data_ptr(),
            meta=self.meta.data_ptr(), error=self.error.data_ptr(),
            window=self.win_desc.data_ptr(), num_pages=self.num_pages,
            num_slots=num_slots, num_layers=num_layers, dim=dim, num_heads=num_heads,
            left=self.left, chunk=self.chunk, page_size=page_size, ring=self.ring,
            dtype=DTYPES[dtype])
        self._desc = d
        h = ctypes.c_void_p()
        check(lib().pk_paged_kv_create(ctypes.byref(d), ctypes.byref(h)), "pk_paged_kv_create")
        self._h = h
        self._lock = threading.Lock()
        self.pending_release: list[int] = []
        self.reset(page_order)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                lib().pk_paged_kv_destroy(h)
            except Exception:
                pass
            self._h = None

    # ------------------------------------------------------------ allocator
    def reset(self, page_order=None):
        """All pages free in ``page_order`` (default 0..num_pages-1)."""
        order = None
        if page_order is not None:
            order = torch.as_tensor(page_order, dtype=torch.int32).to(self.device)
            if order.numel() != self.num_pages:
                raise ValueError("page_order must list every page once")
        self._order = order
        check(lib().pk_pages_reset(self._h, _ptr(order), _stream(self.device)), "pk_pages_reset")
        self.conv.zero_()

    def release_slot(self, slot: int):
        """Queue a finished stream's slot; its pages return to the free ring at
        the start of the next step, before that step's frees and allocations."""
        with self._lock:
            self.pending_release.append(int(slot))

    def begin_step(self, slots: torch.Tensor, lengths: torch.Tensor | None = None,
                   released: torch.Tensor | None = None, relpos=None):
        """Page releases, frees and allocations for one step of ``slots``
        (int32 [B], distinct), then the step's window descriptors for chunks
        of ``lengths`` (int32 [B]; None = full chunks).  ``released`` defaults
        to the queued releases.  ``relpos`` = (layer, query, pos_proj, bias_v,
        out or None): the same launch also computes ``relpos_bd`` of this
        step's rows (pk_pages_begin_step_relpos), which is returned."""
        if released is None:
            with self._lock:
                rel, self.pending_release = self.pending_release, []
            if rel:
                released = torch.tensor(rel, dtype=torch.int32).to(self.device)
        n_rel = 0 if released is None else int(released.numel())
        if relpos is None:
            check(lib().pk_pages_begin_step(self._h, slots.data_ptr(), _ptr(lengths),
                                            int(slots.numel()), _ptr(released) if n_rel else None,
                                            n_rel, _stream(self.device)), "pk_pages_begin_step")
            return None
        layer, query, pos_proj, bias_v, out = relpos
        query, pos_proj, bias_v, out = self._relpos_prep(query, pos_proj, bias_v, out)
        if query.shape[1] != slots.numel():
            raise ValueError("the pre-pass's batch must be the step's batch")
        check(lib().pk_pages_begin_step_relpos(
            self._h, slots.data_ptr(), _ptr(lengths), int(slots.numel()),
            _ptr(released) if n_rel else None, n_rel, layer, query.shape[0], query.data_ptr(),
            query.stride(0), query.stride(1), query.stride(2), pos_proj.data_ptr(),
            pos_proj.stride(0), bias_v.data_ptr(), bias_v.stride(0), out.data_ptr(),
            _stream(self.device)), "pk_pages_begin_step_relpos")
        return out

    def end_step(self, slots: torch.Tensor, lengths: torch.Tensor):
        check(lib().pk_pages_end_step(self._h, slots.data_ptr(), lengths.data_ptr(),
                                      int(slots.numel()), _stream(self.device)),
              "pk_pages_end_step")

    def zero_conv_slot(self, slot: int):
        self.conv[slot].zero_()

    def read_error(self) -> int:
        return int(self.error.item())

    # ------------------------------------------------------------ data path
    def _check_rows(self, t: torch.Tensor, name: str):
        if t.dtype != self.dtype or t.device != self.device:
            raise TypeError(f"{name}: expected {self.dtype} on {self.device}, got {t.dtype} on {t.device}")
        if t.stride(-1) != 1:
            raise ValueError(f"{name}: last dimension must be contiguous")

    def append(self, layer: int, key: torch.Tensor, value: torch.Tensor, slots: torch.Tensor):
        """key/value [B, T, D] (any batch/row strides, e.g. qkv slices) or
        [nl, B, T, D] for layers layer .. layer + nl - 1."""
        if key.dim() == 3:
            key, value = key.unsqueeze(0), value.unsqueeze(0)
        self._check_rows(key, "key")
        self._check_rows(value, "value")
        nl, B, T, D = key.shape
        if T != self.chunk or D != self.dim or value.shape != key.shape or key.stride() != value.stride():
            raise ValueError(f"key/value shape {tuple(key.shape)} vs chunk {self.chunk}, dim {self.dim}")
        check(lib().pk_append_kv(self._h, layer, nl, key.data_ptr(), value.data_ptr(),
                                 key.stride(0), key.stride(1), key.stride(2), slots.data_ptr(), B,
                                 _stream(self.device)), "pk_append_kv")

    def gather(self, layer: int, slots: torch.Tensor, out_k=None, out_v=None):
        B = int(slots.numel())
        shape = (B, self.window, self.dim)
        k = out_k if out_k is not None else torch.empty(shape, dtype=self.dtype, device=self.device)
        v = out_v if out_v is not None else torch.empty(shape, dtype=self.dtype, device=self.device)
        if not (k.is_contiguous() and v.is_contiguous() and tuple(k.shape) == shape):
            raise ValueError("gather outputs must be contiguous [B, W, D]")
        check(lib().pk_gather_window(self._h, layer, slots.data_ptr(), B, k.data_ptr(),
                                     v.data_ptr(), _stream(self.device)), "pk_gather_window")
        return k, v

    def gather_layers(self, layer0: int, num_layers: int, slots: torch.Tensor, out_k=None,
                      out_v=None):
        """gather() of layers layer0 .. layer0 + num_layers - 1 in one launch:
        contiguous [num_layers, B, W, D] outputs."""
        B = int(slots.numel())
        shape = (num_layers, B, self.window, self.dim)
        k = out_k if out_k is not None else torch.empty(shape, dtype=self.dtype, device=self.device)
        v = out_v if out_v is not None else torch.empty(shape, dtype=self.dtype, device=self.device)
        if not (k.is_contiguous() and v.is_contiguous() and tuple(k.shape) == shape):
            raise ValueError("gather_layers outputs must be contiguous [L, B, W, D]")
        check(lib().pk_gather_windows(self._h, layer0, num_layers, slots.data_ptr(), B,
                                      k.data_ptr(), v.data_ptr(), k.stride(0),
                                      _stream(self.device)), "pk_gather_windows")
        return k, v

    @property
    def relpos_bd_cols(self) -> int:
        """Row length of ``relpos_bd``'s output; 0 when this pool's shape has no
        all-stream rel-pos pre-pass."""
        return int(lib().pk_relpos_bd_cols(self._h))

    def _check_attn_inputs(self, query, pos_proj, biases):
        nl, B, T, D = query.shape
        P = 2 * self.window - 1
        if T != self.chunk or D != self.dim:
            raise ValueError(f"query shape {tuple(query.shape)} vs chunk {self.chunk}, dim {self.dim}")
        if pos_proj is not None and (tuple(pos_proj.shape) != (nl, P, D) or not pos_proj[0].is_contiguous()):
            raise ValueError(f"pos_proj must be [{nl}, {P}, {D}] with contiguous rows")
        dh = D // self.num_heads
        for t, n in biases:
            if tuple(t.shape) != (nl, self.num_heads, dh) or not t[0].is_contiguous() or t.dtype != self.dtype:
                raise ValueError(f"{n} must be [{nl}, {self.num_heads}, {dh}] {self.dtype}")

    def _relpos_prep(self, query, pos_proj, bias_v, out):
        if query.dim() == 3:
            query, pos_proj, bias_v = query.unsqueeze(0), pos_proj.unsqueeze(0), bias_v.unsqueeze(0)
        self._check_rows(query, "query")
        self._check_attn_inputs(query, pos_proj, ((bias_v, "bias_v"),))
        nl, B, T, _ = query.shape
        cols = self.relpos_bd_cols
        if cols == 0:
            raise _lib.PKError("relpos_bd: no all-stream pre-pass for this pool's shape")
        shape = (nl, B, self.num_heads, T, cols)
        if out is None:
            out = torch.empty(shape, dtype=torch.float32, device=self.device)
        elif tuple(out.shape) != shape or out.dtype != torch.float32 or not out.is_contiguous():
            raise ValueError(f"out must be contiguous float32 {shape}")
        return query, pos_proj, bias_v, out

    def relpos_bd(self, layer: int, query: torch.Tensor, pos_proj: torch.Tensor,
                  bias_v: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """The rel-pos term (q + pos_bias_v) pos_proj^T of every (layer, stream,
        head, query row), fp32 [nl, B, H, T, relpos_bd_cols], for
        ``attention(..., bd=...)``: one pass over all streams, which share the
        layer's pos_proj rows.  Shapes as in ``attention``."""
        query, pos_proj, bias_v, out = self._relpos_prep(query, pos_proj, bias_v, out)
        nl, B = query.shape[:2]
        check(lib().pk_relpos_bd(
            self._h, layer, nl, query.data_ptr(), query.stride(0), query.stride(1), query.stride(2),
            pos_proj.data_ptr(), pos_proj.stride(0), bias_v.data_ptr(), bias_v.stride(0), B,
            out.data_ptr(), _stream(self.device)), "pk_relpos_bd")
        return out

    def attention(self, layer: int, query: torch.Tensor, pos_proj: torch.Tensor | None,
                  bias_u: torch.Tensor, bias_v: torch.Tensor | None, slots: torch.Tensor,
                  lengths: torch.Tensor, out: torch.Tensor | None = None,
                  key: torch.Tensor | None = None, value: torch.Tensor | None = None,
                  bd: torch.Tensor | None = None, noalloc: bool = False):
        """query [B, T, D] or [nl, B, T, D]; pos_proj [P, D] or [nl, P, D];
        bias_u/v [H, dh] or [nl, H, dh]; lengths int32 [B].  With key/value
        (this step's new rows, the query's shape and strides) the append is
        part of the call.  With ``bd`` (``relpos_bd``'s output for the same
        query) pos_proj and bias_v are not read.  ``noalloc``: for callers that
        must not allocate device memory, pk_paged_attention_noalloc keeps the
        rel-pos term in the library's static 32 MiB device array (larger steps
        are refused; calls overlapping on the GPU race on it, so keep them on
        one stream) and ``out`` must be given.  Returns out with the query's
        leading shape."""
        squeeze = query.dim() == 3
        if squeeze:
            query, bias_u = query.unsqueeze(0), bias_u.unsqueeze(0)
            if bd is None:
                pos_proj, bias_v = pos_proj.unsqueeze(0), bias_v.unsqueeze(0)
            elif bd.dim() == 4:
                bd = bd.unsqueeze(0)
        self._check_rows(query, "query")
        nl, B, T, D = query.shape
        if bd is None:
            self._check_attn_inputs(query, pos_proj, ((bias_u, "bias_u"), (bias_v, "bias_v")))
            if bias_u.stride(0) != bias_v.stride(0):
                raise ValueError("bias_u/bias_v layer strides differ")
        else:
            self._check_attn_inputs(query, None, ((bias_u, "bias_u"),))
            shape = (nl, B, self.num_heads, T, self.relpos_bd_cols)
            if tuple(bd.shape) != shape or bd.dtype != torch.float32 or not bd.is_contiguous():
                raise ValueError(f"bd must be contiguous float32 {shape} (relpos_bd's output)")
        if out is None:
            if noalloc:
                raise ValueError("noalloc=True allocates nothing: pass `out`")
            out = torch.empty((nl, B, T, D), dtype=self.dtype, device=self.device)
        elif out.dim() == 3:
            out = out.unsqueeze(0)
        kp = vp = None
        if key is not None:
            if key.dim() == 3:
                key, value = key.unsqueeze(0), value.unsqueeze(0)
            self._check_rows(key, "key")
            self._check_rows(value, "value")
            if key.shape != query.shape or key.stride() != query.stride() or value.stride() != query.stride():
                raise ValueError("key/value must have the query's shape and strides")
            kp, vp = key.data_ptr(), value.data_ptr()
        if bd is not None:
            check(lib().pk_paged_attention_bd(
                self._h, layer, nl, query.data_ptr(), query.stride(0), query.stride(1),
                query.stride(2), kp, vp, bd.data_ptr(), bias_u.data_ptr(), bias_u.stride(0),
                slots.data_ptr(), lengths.data_ptr(), B, out.data_ptr(), out.stride(0),
                out.stride(1), out.stride(2), _stream(self.device)), "pk_paged_attention_bd")
            return out[0] if squeeze else out
        name = "pk_paged_attention_noalloc" if noalloc else "pk_paged_attention"
        check(getattr(lib(), name)(
            self._h, layer, nl, query.data_ptr(), query.stride(0), query.stride(1),
            query.stride(2), kp, vp, pos_proj.data_ptr(), pos_proj.stride(0), bias_u.data_ptr(),
            bias_v.data_ptr(), bias_u.stride(0), slots.data_ptr(), lengths.data_ptr(), B,
            out.data_ptr(), out.stride(0), out.stride(1), out.stride(2), _stream(self.device)),
            name)
        return out[0] if squeeze else out

    def conv_step(self, layer: int, x: torch.Tensor, weight: torch.Tensor, slots: torch.Tensor,
                  lengths: torch.Tensor, ln_weight=None, ln_bias=None, eps=1e-5, out=None):
        """x: pw-conv1 output [B, T, 2D]; weight [D, kernel] (or [D, 1, kernel]).
        Returns [B, T, D]: the depthwise conv output, or SiLU(LayerNorm(.)) of it
        when ln_weight/ln_bias are given.  Updates the slot conv caches."""
        self._check_rows(x, "x")
        B, T, D2 = x.shape
        if T != self.chunk or D2 != 2 * self.dim:
            raise ValueError(f"x shape {tuple(x.shape)}")
        w = weight.reshape(self.dim, self.conv_kernel)
        if not w.is_contiguous() or w.dtype != self.dtype:
            raise ValueError("conv weight must be contiguous in the pool dtype")
        if out is None:
            out = torch.empty((B, T, self.dim), dtype=self.dtype, device=self.device)
        check(lib().pk_conv_step(
            self.conv.data_ptr(), self.num_slots, self.num_layers, layer, self.dim,
            self.conv_kernel, T, DTYPES[self.dtype], x.data_ptr(), x.stride(0), x.stride(1),
            w.data_ptr(), _ptr(ln_weight), _ptr(ln_bias), float(eps), slots.data_ptr(),
            lengths.data_ptr(), B, out.data_ptr(), self.error.data_ptr(), _stream(self.device)),
            "pk_conv_step")
        return out

    # ------------------------------------------------------------ views
    def counters(self, slots: torch.Tensor):
        """(processed_frames, cache_lengths) int64 of the given slots."""
        m = self.meta.index_select(0, slots.long())
        return (m[:, _lib.META_PROCESSED].long(), m[:, _lib.META_CACHE_LEN].long())
