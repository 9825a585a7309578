"""Torch-tensor wrappers over the C-ABI kernels.

PyTorch supplies device memory and the current stream; every computation is a
call into ``libretree_b200.so``.  Inputs must already be CUDA tensors: there
is no CPU path, and a missing library raises (``retree_b200._lib.load``).
"""

from __future__ import annotations

import ctypes
import threading

import numpy as np
import torch

from . import _lib

_DTYPE_CODE = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}


def _require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("retree_b200 kernels take CUDA tensors (no CPU path)")


def _ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(device=None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class _DeviceState:
    """Per-device scratch and status words (grown on demand, never shrunk)."""

    def __init__(self):
        self.lock = threading.Lock()
        self.bufs: dict = {}

    # Buffers are made outside inference mode: they are updated in place from
    # both inside and outside it (an inference tensor refuses the latter).
    def buffer(self, device, name: str, nbytes: int) -> torch.Tensor:
        key = (torch.device(device).index, name)
        with self.lock:
            b = self.bufs.get(key)
            if b is None or b.numel() < nbytes:
                with torch.inference_mode(False):
                    b = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)
                self.bufs[key] = b
            return b

    def status(self, device) -> torch.Tensor:
        key = (torch.device(device).index, "__status__")
        with self.lock:
            s = self.bufs.get(key)
            if s is None:
                with torch.inference_mode(False):
                    s = torch.zeros(1, dtype=torch.int32, device=device)
                self.bufs[key] = s
            return s


_STATE = _DeviceState()

#: number of kernel launches issued through these wrappers (for launch accounting)
LAUNCHES = 0


def _count(n: int = 1) -> None:
    global LAUNCHES
    LAUNCHES += n


def _nccl_group_up() -> bool:
    import torch.distributed as dist
    return dist.is_available() and dist.is_initialized() and dist.get_backend() == "nccl"


def set_pdl(enabled: bool) -> None:
    """Programmatic dependent launch between the verify-forward kernels (rt_set_pdl).

    It is never turned on in a process with an NCCL process group: a 2-process
    run with NCCL collectives between dependent-launched kernels stalled, with
    no cause found, so the two are kept apart (``pdl_guard``).
    """
    if enabled and _nccl_group_up():
        raise RuntimeError("programmatic dependent launch stays off in a process with an NCCL process group")
    _lib.load().rt_set_pdl(int(bool(enabled)))


def pdl_guard() -> None:
    """Turn programmatic dependent launch off if this process has an NCCL process group."""
    if _nccl_group_up():
        _lib.load().rt_set_pdl(0)


def pdl_enabled() -> bool:
    return bool(_lib.load().rt_pdl_enabled())


def status_tensor(device) -> torch.Tensor:
    """The device status word the kernels of this process report into."""
    return _STATE.status(device)


def check_device_status(device, reset: bool = True) -> None:
    """Synchronise on the status word and raise if a kernel reported an error."""
    s = _STATE.status(device)
    code = int(s.item())
    if reset and code:
        s.zero_()
    if code:
        raise RuntimeError(f"retree_b200 kernel reported: {_lib.status_string(code)}")


# ---------------------------------------------------------------------------
# KV cache
# ---------------------------------------------------------------------------
def kv_compact(tensors, past_length: int, keep: torch.Tensor, cur_length: int | None = None,
               n_keep_dev: torch.Tensor | None = None, n_keep: int | None = None,
               past_len_dev: torch.Tensor | None = None) -> None:
    """In-place compaction of appended rows (ddtree.py:666-731 semantics).

    ``tensors``: one ``[..., S, D]`` tensor or a list of them.  All leading
    dims of a tensor are folded into one head axis when their strides allow
    (a whole ``[layers*2, heads, S, D]`` slab then moves in ONE launch).
    ``keep``: int64 CUDA tensor of window-relative indices; ``n_keep_dev``
    (int32[1], optional) supplies the count at run time.
    """
    lib = _lib.load()
    group = [tensors] if isinstance(tensors, torch.Tensor) else list(tensors)
    if not group:
        return
    _require_cuda(keep, *group)
    if keep.dtype != torch.int64:
        raise RuntimeError("keep_current_indices must have dtype torch.long")
    nk = int(keep.numel()) if n_keep is None else int(n_keep)
    for t in group:
        if t.dim() < 2:
            raise RuntimeError("cache_tensor must have rank >= 2")
        seq = t.shape[-2]
        if past_len_dev is None and (past_length < 0 or past_length > seq):
            raise RuntimeError("past_length exceeds cache sequence length")
        cur = (seq - past_length) if cur_length is None else int(cur_length)
        if cur <= 0:
            continue
        if t.stride(-1) != 1:
            raise RuntimeError("cache rows must be contiguous")
        try:
            v = t.view(-1, seq, t.shape[-1])
        except RuntimeError:
            kv_compact(list(t.unbind(0)), past_length, keep, cur_length, n_keep_dev, n_keep, past_len_dev)
            continue
        es = v.element_size()
        rc = lib.rt_kv_compact(None, v.data_ptr(), 1, 0, v.shape[0], v.stride(0) * es, v.stride(1) * es,
                               v.shape[2] * es, int(past_length), _ptr(past_len_dev), cur, keep.data_ptr(), nk,
                               _ptr(n_keep_dev), _STATE.status(t.device).data_ptr(), _stream(t.device))
        _lib.check(rc, "rt_kv_compact")
        _count()


def kv_append(k_cache: torch.Tensor, v_cache: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
              offset: int = 0, offset_dev: torch.Tensor | None = None) -> None:
    """Write ``[heads, n, D]`` new rows at ``offset`` of ``[heads, cap, D]`` caches (views allowed)."""
    lib = _lib.load()
    _require_cuda(k_cache, v_cache, k_new, v_new)
    k_cache, v_cache = _as3(k_cache), _as3(v_cache)
    k_new, v_new = _as3(k_new), _as3(v_new)
    if k_cache.stride() != v_cache.stride():
        raise RuntimeError("K and V caches must share strides")
    if k_new.stride() != v_new.stride():
        k_new, v_new = k_new.contiguous(), v_new.contiguous()
    es = k_cache.element_size()
    heads, n, d = k_new.shape
    rc = lib.rt_kv_append(k_cache.data_ptr(), v_cache.data_ptr(), k_cache.stride(0) * es, k_cache.stride(1) * es,
                          k_new.data_ptr(), v_new.data_ptr(), k_new.stride(0) * es, k_new.stride(1) * es, heads, n,
                          d * es, k_cache.shape[1], int(offset), _ptr(offset_dev),
                          _STATE.status(k_cache.device).data_ptr(), _stream(k_cache.device))
    _lib.check(rc, "rt_kv_append")
    _count()


def _as3(t: torch.Tensor) -> torch.Tensor:
    if t.dim() == 4:
        if t.shape[0] != 1:
            raise RuntimeError("batch size 1 only")
        t = t[0]
    if t.dim() != 3 or t.stride(-1) != 1:
        raise RuntimeError("expected [heads, seq, head_dim] with contiguous head_dim")
    return t


# ---------------------------------------------------------------------------
# Tree-verify attention
# ---------------------------------------------------------------------------
def tree_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask_bits: torch.Tensor, prefix_len: int,
                   scale: float | None = None, out: torch.Tensor | None = None, num_splits: int = 0,
                   path: int = 0, prefix_len_dev: torch.Tensor | None = None,
                   kv_capacity: int | None = None) -> torch.Tensor:
    """Masked GQA attention of n tree nodes over ``[prefix ; tree block]``.

    q: ``[n, Hq, D]`` or HF's ``[1, Hq, n, D]``; k, v: ``[Hkv, S, D]`` or
    ``[1, Hkv, S, D]`` (rows ``[0, prefix_len + n)`` are used);
    mask_bits: int32 ``[n, W]`` ancestor bits of the tree block.
    Returns ``out`` ``[n, Hq, D]`` bf16 (HF's ``[1, n, Hq, D]`` after unsqueeze).
    """
    lib = _lib.load()
    _require_cuda(q, k, v, mask_bits)
    if q.dim() == 4:
        if q.shape[0] != 1:
            raise RuntimeError("batch size 1 only")
        q = q[0].transpose(0, 1)  # [n, Hq, D] view
    k, v = _as3(k), _as3(v)
    if k.stride() != v.stride():
        raise RuntimeError("K and V must share strides")
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16:
        raise RuntimeError("tree attention runs on bf16 q/k/v")
    n, hq, d = q.shape
    hkv = k.shape[0]
    if out is None:
        out = torch.empty((n, hq, d), dtype=torch.bfloat16, device=q.device)
    es = 2
    mask_bits = mask_bits if mask_bits.dim() == 2 else mask_bits.reshape(n, -1)
    if mask_bits.stride(-1) != 1:
        mask_bits = mask_bits.contiguous()
    words = mask_bits.stride(0)
    scale = d ** -0.5 if scale is None else float(scale)
    cap = k.shape[1] if kv_capacity is None else int(kv_capacity)
    splits, merged = attn_plan(n, hq, hkv, int(prefix_len), num_splits, path)
    ws_bytes = 0 if merged else lib.rt_tree_attn_workspace_size(n, hq, hkv, d, int(prefix_len), splits)
    ws = _STATE.buffer(q.device, "attn_ws", ws_bytes) if ws_bytes else None
    rc = lib.rt_tree_attn(q.data_ptr(), q.stride(0) * es, q.stride(1) * es, k.data_ptr(), v.data_ptr(),
                          k.stride(0) * es, k.stride(1) * es, cap, out.data_ptr(), out.stride(0) * es,
                          out.stride(1) * es, mask_bits.data_ptr(), words, n, int(prefix_len),
                          _ptr(prefix_len_dev), hq, hkv, d, scale, splits, path, _ptr(ws), ws_bytes,
                          _STATE.status(q.device).data_ptr(), _stream(q.device))
    _lib.check(rc, "rt_tree_attn")
    _count(2 if ws_bytes else 1)  # the combine launch runs only when the partials go through the workspace
    return out


def attn_plan(n: int, num_q_heads: int, num_kv_heads: int, prefix_len: int, num_splits: int = 0,
              path: int = 0) -> tuple[int, bool]:
    """(key splits, merged in the kernel) of an rt_tree_attn launch of this shape (rt_tree_attn_plan)."""
    sp, mg = ctypes.c_int(0), ctypes.c_int(0)
    _lib.check(_lib.load().rt_tree_attn_plan(n, num_q_heads, num_kv_heads, int(prefix_len), int(num_splits), int(path),
                                             ctypes.byref(sp), ctypes.byref(mg), None), "rt_tree_attn_plan")
    return sp.value, bool(mg.value)


def default_splits(n: int, num_q_heads: int, num_kv_heads: int, prefix_len: int) -> int:
    """Key splits rt_tree_attn picks for this shape (one wave of CTAs)."""
    return int(_lib.load().rt_tree_attn_default_splits(n, num_q_heads, num_kv_heads, int(prefix_len)))


def mask_from_dense(dense: torch.Tensor, col0: int, n: int, words: int | None = None) -> torch.Tensor:
    """Packed bits of the tree block of a dense additive mask (0 = visible)."""
    lib = _lib.load()
    _require_cuda(dense)
    d2 = dense.reshape(-1, dense.shape[-1]) if dense.dim() > 2 else dense
    if d2.stride(-1) != 1:
        raise RuntimeError("dense mask rows must be contiguous")
    w = (n + 31) // 32 if words is None else words
    bits = torch.empty((n, w), dtype=torch.int32, device=dense.device)
    rc = lib.rt_mask_from_dense(d2.data_ptr(), _DTYPE_CODE[d2.dtype], d2.stride(0), int(col0), n, bits.data_ptr(),
                                w, _stream(dense.device))
    _lib.check(rc, "rt_mask_from_dense")
    _count()
    return bits


# ---------------------------------------------------------------------------
# Draft top-k and tree construction
# ---------------------------------------------------------------------------
def draft_topk(logits: torch.Tensor, k: int, out=None):
    """``(top_logp f32[R,k], top_ids i64[R,k], log_z f32[R])`` of ``[R, V]`` logits on the device."""
    lib = _lib.load()
    _require_cuda(logits)
    if logits.dim() != 2 or logits.stride(-1) != 1:
        raise RuntimeError("logits must be [rows, vocab] with contiguous rows")
    rows, vocab = logits.shape
    dev = logits.device
    if out is None:
        out = (torch.empty((rows, k), dtype=torch.float32, device=dev),
               torch.empty((rows, k), dtype=torch.int64, device=dev),
               torch.empty((rows,), dtype=torch.float32, device=dev))
    ws_bytes = lib.rt_draft_topk_workspace_size(rows, vocab, k)
    ws = _STATE.buffer(dev, "topk_ws", ws_bytes)
    rc = lib.rt_draft_topk(logits.data_ptr(), _DTYPE_CODE[logits.dtype], logits.stride(0), rows, vocab, k,
                           out[0].data_ptr(), out[1].data_ptr(), out[2].data_ptr(), ws.data_ptr(), ws_bytes,
                           _stream(dev))
    _lib.check(rc, "rt_draft_topk")
    _count(2)
    return out


STRATEGY_CODE = {"heap": 0, "ngram": 1, "rank_gated_ngram": 2}

_LOG1P_CACHE: dict = {}


def log1p_table(device, n: int) -> torch.Tensor:
    """``np.log1p(c)`` for c = 0..n as binary64 on ``device`` (the reference's bonus base)."""
    key = (torch.device(device).index, n)
    t = _LOG1P_CACHE.get(key)
    if t is None:
        t = torch.from_numpy(np.log1p(np.arange(n + 1, dtype=np.float64))).to(device)
        _LOG1P_CACHE[key] = t
    return t


def tree_build(top_logp: torch.Tensor, top_ids: torch.Tensor, budget: int, strategy: str, params,
               ctx: torch.Tensor | None = None, ctx_len_dev: torch.Tensor | None = None, ctx_len: int | None = None,
               out: dict | None = None, root: int = -1, root_dev=None, start: int = 0, start_dev=None,
               mask_words: int | None = None) -> dict:
    """Best-first expansion on the device; returns a dict of device tensors.

    Keys: tokens i64[budget], depths i64[budget], parents i32[budget+1],
    mask i32[budget+1, W], count i32[1], verify_ids i64[budget+1],
    verify_pos i64[budget+1].  ``params``: oracle-compatible n-gram knobs
    (``max_n, beta, rank_cap, min_count, context_window, use_log_count,
    longer_weight, max_token_bonus``).
    """
    lib = _lib.load()
    _require_cuda(top_logp, top_ids, ctx)
    dev = top_logp.device
    rows, k = top_logp.shape
    code = STRATEGY_CODE[strategy]
    w = (budget + 1 + 31) // 32 if mask_words is None else mask_words
    if out is None:
        out = dict(
            tokens=torch.empty(max(budget, 1), dtype=torch.int64, device=dev),
            depths=torch.empty(max(budget, 1), dtype=torch.int64, device=dev),
            parents=torch.empty(budget + 1, dtype=torch.int32, device=dev),
            mask=torch.empty((budget + 1, w), dtype=torch.int32, device=dev),
            count=torch.empty(1, dtype=torch.int32, device=dev),
            verify_ids=torch.empty(budget + 1, dtype=torch.int64, device=dev),
            verify_pos=torch.empty(budget + 1, dtype=torch.int64, device=dev),
        )
    max_n = int(params.max_n) if code else 2
    ow_vals = [float(params.longer_weight ** max(0, n - 2)) for n in range(2, max_n + 1)]
    ow = (ctypes.c_double * max(len(ow_vals), 1))(*ow_vals)
    window = int(params.context_window)
    if ctx is not None:
        clen = int(ctx.numel()) if ctx_len is None else int(ctx_len)
    else:
        clen = 0
    # one table per window size (not per context length), so it is uploaded once
    table_n = window if window > 0 else max(clen, 1)
    table = log1p_table(dev, max(table_n, 1) + 1)
    rc = lib.rt_tree_build(
        top_logp.data_ptr(), top_ids.data_ptr(), rows, k, int(budget), code, _ptr(ctx), clen, _ptr(ctx_len_dev),
        window, max_n, float(params.beta), int(params.rank_cap), int(params.min_count), int(bool(params.use_log_count)),
        ctypes.addressof(ow), float(params.max_token_bonus), table.data_ptr(), int(table.numel()),
        out["tokens"].data_ptr(), out["depths"].data_ptr(), out["parents"].data_ptr(), out["mask"].data_ptr(), w,
        out["count"].data_ptr(), _ptr(out.get("verify_ids")), _ptr(out.get("verify_pos")), int(root), _ptr(root_dev),
        int(start), _ptr(start_dev), _STATE.status(dev).data_ptr(), _stream(dev))
    _lib.check(rc, "rt_tree_build")
    _count()
    out["_keep_alive"] = (ow, table)
    return out


def tree_walk(parents: torch.Tensor, tokens: torch.Tensor, posterior: torch.Tensor, count: int | None = None,
              count_dev: torch.Tensor | None = None, out: dict | None = None, verify_ids=None, output_ids=None,
              start_dev=None) -> dict:
    """Exact walk on the device; returns ``accepted`` i64[n], ``accepted_len`` i32[1], ``next_token`` i64[1]."""
    lib = _lib.load()
    _require_cuda(parents, tokens, posterior)
    dev = parents.device
    n = parents.numel()
    if out is None:
        out = dict(accepted=torch.empty(n, dtype=torch.int64, device=dev),
                   accepted_len=torch.empty(1, dtype=torch.int32, device=dev),
                   next_token=torch.empty(1, dtype=torch.int64, device=dev))
    cnt = (n - 1) if count is None else int(count)
    post = posterior.reshape(-1)
    if post.dtype != torch.int64:
        post = post.to(torch.int64)
    rc = lib.rt_tree_walk(parents.data_ptr(), tokens.data_ptr(), cnt, _ptr(count_dev), post.data_ptr(),
                          out["accepted"].data_ptr(), out["accepted_len"].data_ptr(), out["next_token"].data_ptr(),
                          _ptr(verify_ids), _ptr(output_ids), 0 if output_ids is None else output_ids.numel(),
                          _ptr(start_dev), _STATE.status(dev).data_ptr(), _stream(dev))
    _lib.check(rc, "rt_tree_walk")
    _count()
    return out


__all__ = ["kv_compact", "kv_append", "tree_attention", "mask_from_dense", "draft_topk", "tree_build",
           "tree_walk", "log1p_table", "status_tensor", "check_device_status", "STRATEGY_CODE"]


# ---------------------------------------------------------------------------
# Elementwise stages of the verify forward (retree_b200.fused)
# ---------------------------------------------------------------------------
def _rows_bf16(t: torch.Tensor, name: str) -> None:
    if t.dtype != torch.bfloat16 or not t.is_contiguous():
        raise RuntimeError(f"{name} must be a contiguous bf16 tensor")


def embed_rmsnorm(ids: torch.Tensor, table: torch.Tensor, weight: torch.Tensor, eps: float,
                  residual: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """``residual = table[ids]``; ``out = rmsnorm(residual) * weight`` (bf16, rows = ids.numel())."""
    _require_cuda(ids, table, weight, residual, out)
    for t, nm in ((table, "table"), (weight, "weight"), (residual, "residual"), (out, "out")):
        _rows_bf16(t, nm)
    if ids.dtype != torch.int64 or not ids.is_contiguous():
        raise RuntimeError("ids must be contiguous int64")
    rows, hidden = ids.numel(), table.shape[-1]
    _lib.check(_lib.load().rt_embed_rmsnorm(ids.data_ptr(), table.data_ptr(), table.shape[0], residual.data_ptr(),
                                            weight.data_ptr(), out.data_ptr(), rows, hidden, float(eps),
                                            status_tensor(ids.device).data_ptr(), _stream(ids.device)),
               "rt_embed_rmsnorm")
    _count()
    return out


def add_rmsnorm(delta: torch.Tensor | None, residual: torch.Tensor, weight: torch.Tensor, eps: float,
                out: torch.Tensor) -> torch.Tensor:
    """``residual += delta`` (bf16 rounding), ``out = rmsnorm(residual) * weight``; delta may be None."""
    _require_cuda(delta, residual, weight, out)
    for t, nm in ((residual, "residual"), (weight, "weight"), (out, "out")) + (((delta, "delta"),) if delta is not None else ()):
        _rows_bf16(t, nm)
    hidden = residual.shape[-1]
    rows = residual.numel() // hidden
    _lib.check(_lib.load().rt_add_rmsnorm(_ptr(delta), residual.data_ptr(), weight.data_ptr(), out.data_ptr(), rows,
                                          hidden, float(eps), _stream(residual.device)), "rt_add_rmsnorm")
    _count()
    return out


def qk_norm_rope_append(qkv: torch.Tensor, num_q_heads: int, num_kv_heads: int, q_norm_w, k_norm_w, eps: float,
                        cos_table: torch.Tensor, sin_table: torch.Tensor, positions: torch.Tensor,
                        q_out: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, offset: int = 0,
                        offset_dev: torch.Tensor | None = None) -> torch.Tensor:
    """Per-head q/k RMSNorm + rotary embedding; q to ``q_out [n, Hq, 128]``, k/v appended to the cache.

    ``k_cache``/``v_cache`` are ``[Hkv, capacity, 128]`` views with unit inner
    stride; rows land at ``offset`` (+ ``offset_dev[0]`` when given).
    """
    _require_cuda(qkv, cos_table, sin_table, positions, q_out, k_cache, v_cache, q_norm_w, k_norm_w, offset_dev)
    _rows_bf16(qkv, "qkv")
    _rows_bf16(q_out, "q_out")
    n = positions.numel()
    if qkv.numel() != n * (num_q_heads + 2 * num_kv_heads) * 128:
        raise RuntimeError("qkv does not hold n rows of (Hq + 2 Hkv) heads of 128")
    if positions.dtype != torch.int64 or not positions.is_contiguous():
        raise RuntimeError("positions must be contiguous int64")
    if k_cache.stride() != v_cache.stride() or k_cache.stride(-1) != 1 or k_cache.shape[0] != num_kv_heads:
        raise RuntimeError("k_cache/v_cache must be [Hkv, capacity, 128] views with equal strides")
    es = k_cache.element_size()
    _lib.check(_lib.load().rt_qk_norm_rope_append(
        qkv.data_ptr(), n, num_q_heads, num_kv_heads, 128, _ptr(q_norm_w), _ptr(k_norm_w), float(eps),
        cos_table.data_ptr(), sin_table.data_ptr(), cos_table.shape[0], positions.data_ptr(), q_out.data_ptr(),
        k_cache.data_ptr(), v_cache.data_ptr(), k_cache.stride(0) * es, k_cache.stride(1) * es, k_cache.shape[1],
        int(offset), _ptr(offset_dev), status_tensor(qkv.device).data_ptr(), _stream(qkv.device)),
        "rt_qk_norm_rope_append")
    _count()
    return q_out


def silu_mul(gate_up: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """``out = silu(gate) * up`` over ``gate_up = [gate | up]`` rows (bf16)."""
    _require_cuda(gate_up, out)
    _rows_bf16(gate_up, "gate_up")
    _rows_bf16(out, "out")
    inter = out.shape[-1]
    rows = out.numel() // inter
    if gate_up.numel() != 2 * rows * inter:
        raise RuntimeError("gate_up must hold [rows, 2 * inter]")
    _lib.check(_lib.load().rt_silu_mul(gate_up.data_ptr(), out.data_ptr(), rows, inter, _stream(out.device)),
               "rt_silu_mul")
    _count()
    return out


# ---------------------------------------------------------------------------
# tcgen05 projections with fused epilogues (rt_linear)
# ---------------------------------------------------------------------------
def linear_supported(m: int, n_out: int, k: int, epilogue: int = 0) -> bool:
    """Whether rt_linear takes this projection shape."""
    return _lib.load().rt_linear_check(m, n_out, k, epilogue) == _lib.RT_OK


def linear_plan(m: int, n_out: int, k: int, epilogue: int = 0) -> dict:
    """The launch rt_linear makes for a shape on the current device (K splits, ring stages, smem)."""
    vals = [ctypes.c_int(0) for _ in range(3)]
    _lib.check(_lib.load().rt_linear_plan(m, n_out, k, epilogue, *[ctypes.addressof(v) for v in vals]),
               "rt_linear_plan")
    return dict(splits=vals[0].value, stages=vals[1].value, smem=vals[2].value)


def linear(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None, epilogue: int = 0,
           qkv: dict | None = None) -> torch.Tensor | None:
    """``x [m, k] @ w[n_out, k]^T`` on tcgen05 with an optional fused epilogue (bf16).

    epilogue 0: ``out [m, n_out]``; 1 (w = [gate; up]): ``out [m, n_out/2] =
    silu(gate) * up``; 2 (w = [Wq; Wk; Wv]): head norms + rotary, q to
    ``qkv['q_out']``, k/v into the cache (keys of ``qkv`` as in
    ``qk_norm_rope_append``: num_q_heads, num_kv_heads, q_norm, k_norm, eps,
    cos, sin, positions, q_out, k_cache, v_cache, offset, offset_dev).
    """
    lib = _lib.load()
    _require_cuda(x, w, out)
    if x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16 or x.dim() != 2 or x.stride(-1) != 1:
        raise RuntimeError("linear takes bf16 x [m, k] with unit inner stride and bf16 w [n_out, k]")
    if not w.is_contiguous():
        raise RuntimeError("linear weights must be contiguous")
    m, k = x.shape
    n_out = w.shape[0]
    if w.shape[1] != k:
        raise RuntimeError("weight / input inner dimensions differ")
    dev = x.device
    if lib.rt_linear_check(m, n_out, k, epilogue) != _lib.RT_OK:
        raise RuntimeError(f"rt_linear does not take m={m}, n_out={n_out}, k={k}")
    epi = None
    keep = []
    if epilogue == _lib.RT_EPI_QKV_ROPE:
        kc, vc = qkv["k_cache"], qkv["v_cache"]
        es = kc.element_size()
        epi = _lib.QkvEpilogue(qkv["num_q_heads"], qkv["num_kv_heads"], _ptr(qkv.get("q_norm")),
                               _ptr(qkv.get("k_norm")), float(qkv["eps"]), qkv["cos"].data_ptr(),
                               qkv["sin"].data_ptr(), qkv["cos"].shape[0], qkv["positions"].data_ptr(),
                               qkv["q_out"].data_ptr(), kc.data_ptr(), vc.data_ptr(), kc.stride(0) * es,
                               kc.stride(1) * es, kc.shape[1], int(qkv.get("offset", 0)),
                               _ptr(qkv.get("offset_dev")))
        keep.append(epi)
        out_ptr, ld = None, 0
    else:
        if out is None:
            width = n_out // 2 if epilogue == _lib.RT_EPI_SILU_MUL else n_out
            out = torch.empty((m, width), dtype=torch.bfloat16, device=dev)
        if out.dtype != torch.bfloat16 or out.stride(-1) != 1:
            raise RuntimeError("linear output must be bf16 with unit inner stride")
        out_ptr, ld = out.data_ptr(), out.stride(0)
    rc = lib.rt_linear(x.data_ptr(), x.stride(0), m, k, w.data_ptr(), n_out, int(epilogue), out_ptr, ld,
                       ctypes.addressof(epi) if epi is not None else None, status_tensor(dev).data_ptr(),
                       _stream(dev))
    _lib.check(rc, "rt_linear")
    _count()
    return out


# ---------------------------------------------------------------------------
# Target-gated sibling-recovery walk (rt_recovery_walk)
# ---------------------------------------------------------------------------
def linear_argmax(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor, index: torch.Tensor) -> torch.Tensor:
    """``out [m, n_out] = x @ w^T`` (rt_linear) and ``index [m]`` = each row's argmax (first largest; NaN
    largest) from the same launch (rt_linear_argmax): the temperature-0 posterior without a pass over
    the logits."""
    _require_cuda(x, w, out, index)
    if x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16 or x.dim() != 2 or x.stride(-1) != 1:
        raise RuntimeError("linear_argmax takes bf16 x [m, k] with unit inner stride")
    if not w.is_contiguous() or out.dtype != torch.bfloat16 or out.stride(-1) != 1:
        raise RuntimeError("linear_argmax: contiguous bf16 weights, bf16 out with unit inner stride")
    if index.dtype != torch.int64 or not index.is_contiguous() or index.numel() < x.shape[0]:
        raise RuntimeError("index must be contiguous int64 [m]")
    m, k = x.shape
    n_out = w.shape[0]
    keys = _STATE.buffer(x.device, "argmax_keys", max(8 * m, 256))
    _lib.check(_lib.load().rt_linear_argmax(x.data_ptr(), x.stride(0), m, k, w.data_ptr(), n_out, out.data_ptr(),
                                            out.stride(0), keys.data_ptr(), index.data_ptr(),
                                            status_tensor(x.device).data_ptr(), _stream(x.device)),
               "rt_linear_argmax")
    _count(2)  # the projection and the index conversion (the key reset is a memset)
    return index


def recovery_walk(parents: torch.Tensor, tokens: torch.Tensor, posterior: torch.Tensor, logits: torch.Tensor,
                  table: tuple, params: dict, count: int | None = None, count_dev: torch.Tensor | None = None,
                  stop_ids: torch.Tensor | None = None, log: tuple | None = None, out: dict | None = None,
                  verify_ids: torch.Tensor | None = None, output_ids: torch.Tensor | None = None,
                  start_dev: torch.Tensor | None = None) -> dict:
    """ReTree's recovery walk on the device.

    ``table`` = (keys int64[cap], prior int32[cap], online int32[cap]) of
    ``recovery_device.RecoveryTable``; ``params`` = gate_threshold,
    freq_threshold, rescue_top_k, record_top_k, online_update; ``log`` =
    (pairs int32[cap, 2], count int32[1]) or None; ``stop_ids`` int64 or None
    (no stop set).  Returns ``out`` with accepted / accepted_len / next_token /
    rescued.
    """
    _require_cuda(parents, tokens, posterior, logits, stop_ids, verify_ids, output_ids, start_dev, *table)
    dev = parents.device
    n_max = parents.numel()
    cnt = n_max - 1 if count is None else int(count)
    if logits.dtype not in (torch.float32, torch.bfloat16) or logits.dim() != 2 or logits.stride(-1) != 1:
        raise RuntimeError("logits must be [nodes, vocab] fp32 or bf16 with contiguous rows")
    if out is None:
        out = dict(accepted=torch.zeros(n_max, dtype=torch.int64, device=dev),
                   accepted_len=torch.zeros(1, dtype=torch.int32, device=dev),
                   next_token=torch.zeros(1, dtype=torch.int64, device=dev),
                   rescued=torch.zeros(1, dtype=torch.int32, device=dev))
    keys, prior, online = table
    log_pairs, log_count = (None, None) if log is None else log
    rc = _lib.load().rt_recovery_walk(
        parents.data_ptr(), _ptr(tokens), cnt, _ptr(count_dev), posterior.data_ptr(), logits.data_ptr(),
        logits.stride(0), 0 if logits.dtype == torch.float32 else 1, logits.shape[1],
        float(params.get("gate_threshold", 0.01)), int(params.get("freq_threshold", 6)),
        int(params.get("rescue_top_k", 8)), int(params.get("record_top_k", 8)),
        int(bool(params.get("online_update", True))), _ptr(stop_ids),
        0 if stop_ids is None else stop_ids.numel(), keys.data_ptr(), prior.data_ptr(), online.data_ptr(),
        keys.numel(), _ptr(log_pairs), _ptr(log_count), 0 if log_pairs is None else log_pairs.shape[0],
        out["accepted"].data_ptr(), out["accepted_len"].data_ptr(), out["next_token"].data_ptr(),
        out["rescued"].data_ptr(), _ptr(verify_ids), _ptr(output_ids),
        0 if output_ids is None else output_ids.numel(), _ptr(start_dev), status_tensor(dev).data_ptr(),
        _stream(dev))
    _lib.check(rc, "rt_recovery_walk")
    _count()
    return out
