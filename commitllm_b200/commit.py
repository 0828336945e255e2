"""Host runtime over libvcommit: device buffers, streams and descriptors.

Everything here is plumbing around the C ABI (``include/vcommit.h``): torch
supplies device memory and streams, the hashing runs in the library's CUDA
kernels.  Tensors on a CUDA device are read in place; host arrays (numpy,
bytes, CPU tensors) are copied to the device first.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import List, Optional, Sequence

import numpy as np
import torch

from . import _lib
from ._lib import KvDesc, TraceDesc, check, lib

_DTYPES = {torch.bfloat16: _lib.VC_DTYPE_BF16, torch.float32: _lib.VC_DTYPE_F32,
           torch.float64: _lib.VC_DTYPE_F64, torch.uint16: _lib.VC_DTYPE_BF16,
           torch.int16: _lib.VC_DTYPE_BF16}


def _require_cuda(t: torch.Tensor, name: str) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")


def _i32(seq) -> ctypes.Array:
    arr = (ctypes.c_int32 * max(len(seq), 1))()
    for i, v in enumerate(seq):
        arr[i] = int(v)
    return arr


def _i64(seq) -> ctypes.Array:
    arr = (ctypes.c_int64 * max(len(seq), 1))()
    for i, v in enumerate(seq):
        arr[i] = int(v)
    return arr


def _ptrs(seq) -> ctypes.Array:
    arr = (ctypes.c_void_p * max(len(seq), 1))()
    for i, v in enumerate(seq):
        arr[i] = v
    return arr


class _DevView:
    """__cuda_array_interface__ view of library-owned device memory."""

    def __init__(self, ptr: int, nbytes: int, owner):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3, "strides": None}
        self._owner = owner


class Context:
    """A libvcommit context bound to one device and one CUDA stream.

    Calls are stream-ordered on ``self.stream`` (torch's current stream of the
    device by default).  Use one context per stream.
    """

    def __init__(self, device: Optional[int] = None, stream: Optional[torch.cuda.Stream] = None):
        if not torch.cuda.is_available():
            raise RuntimeError("commitllm_b200 needs a CUDA device")
        self.device = torch.cuda.current_device() if device is None else int(device)
        self.stream = stream if stream is not None else torch.cuda.current_stream(self.device)
        self._h = ctypes.c_void_p()
        self._side = None
        check(lib().vc_ctx_create(self.device, ctypes.c_void_p(self.stream.cuda_stream), ctypes.byref(self._h)))

    def side(self) -> "Context":
        """A second context of this device on its own stream, for work that
        should overlap this context's (created on first use, then kept)."""
        if self._side is None:
            self._side = Context(self.device, torch.cuda.Stream(self.device))
        return self._side

    def fork(self) -> "Context":
        """The side context, ordered after everything queued on this one so far."""
        s = self.side()
        s.stream.wait_stream(self.stream)
        return s

    def join(self, other: "Context") -> None:
        """Order this context's later work after everything queued on ``other``."""
        self.stream.wait_stream(other.stream)

    @property
    def handle(self) -> ctypes.c_void_p:
        if not self._h:
            raise RuntimeError("context is closed")
        return self._h

    def sync(self, timeout_ms: int = 0) -> None:
        check(lib().vc_ctx_sync(self.handle, int(timeout_ms)))

    def close(self) -> None:
        if self._side is not None:
            self._side.close()
            self._side = None
        if self._h:
            lib().vc_ctx_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def empty(self, *shape, dtype=torch.uint8) -> torch.Tensor:
        # Allocated on this context's stream, so the caching allocator only
        # reuses the block for work ordered after ours.
        with torch.cuda.stream(self.stream):
            return torch.empty(*shape, dtype=dtype, device=f"cuda:{self.device}")

    def to_device(self, x, dtype=None) -> torch.Tensor:
        """Copy host data (numpy / bytes / CPU tensor) to this device; CUDA tensors pass through."""
        if isinstance(x, torch.Tensor):
            t = x
        elif isinstance(x, (bytes, bytearray, memoryview)):
            t = torch.frombuffer(bytearray(x), dtype=torch.uint8)
        else:
            a = np.ascontiguousarray(x)
            if not a.flags.writeable:
                a = a.copy()
            t = torch.from_numpy(a)
        if dtype is not None and t.dtype != dtype:
            t = t.to(dtype)
        if not t.is_cuda or t.device.index != self.device:
            with torch.cuda.stream(self.stream):
                t = t.to(f"cuda:{self.device}", non_blocking=False)
        return t.contiguous()


class TreeSet:
    """Device-resident Merkle trees (every node, for openings)."""

    def __init__(self, ctx: Context, handle: ctypes.c_void_p):
        self.ctx = ctx
        self._h = handle

    def __len__(self) -> int:
        return lib().vc_tree_set_count(self._h)

    def tree_shape(self, tree: int):
        n = ctypes.c_int64()
        pad = ctypes.c_int64()
        ptr = ctypes.c_void_p()
        check(lib().vc_tree_nodes(self._h, int(tree), ctypes.byref(ptr), ctypes.byref(n), ctypes.byref(pad)))
        return ptr.value, n.value, pad.value

    def nodes(self, tree: int) -> torch.Tensor:
        """The tree's node array ``[2*padded-1, 32]`` (merkle.rs MerkleTree.nodes), a device view."""
        ptr, _n, pad = self.tree_shape(tree)
        nbytes = (2 * pad - 1) * 32
        return torch.as_tensor(_DevView(ptr, nbytes, self), device=f"cuda:{self.ctx.device}").view(-1, 32)

    def prove(self, trees: Sequence[int], leaves: Sequence[int]):
        """merkle::prove for each (tree, leaf): returns (siblings uint8 [n, depth, 32] on device, depths)."""
        n = len(trees)
        if n != len(leaves):
            raise ValueError("trees and leaves differ in length")
        max_depth = 0
        for t in set(int(x) for x in trees):
            _, _, pad = self.tree_shape(t)
            max_depth = max(max_depth, pad.bit_length() - 1)
        sib = self.ctx.empty(max(n, 1), max(max_depth, 1), 32)
        depth = (ctypes.c_int32 * max(n, 1))()
        leaf_arr = (ctypes.c_uint32 * max(n, 1))(*[int(x) & 0xFFFFFFFF for x in leaves])
        for x in leaves:
            if int(x) < 0 or int(x) > 0xFFFFFFFF:
                raise _lib.VcValueError(_lib.VC_ERANGE, f"leaf index {x} out of range")
        check(lib().vc_prove(self.ctx.handle, self._h, n, _i32(trees), leaf_arr, ctypes.c_void_p(sib.data_ptr()),
                             max_depth, depth))
        return sib[:n], [depth[i] for i in range(n)]

    def free(self) -> None:
        if self._h:
            lib().vc_tree_set_free(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


# ---------------------------------------------------------------------------
# KV cache commitment
# ---------------------------------------------------------------------------

@dataclass
class KvCacheView:
    """Where one layer range of K/V rows lives on the device.

    ``k_layers[l]`` / ``v_layers[l]`` are CUDA tensors of one dtype (bf16, f32
    or f64; raw bf16 bits as int16/uint16 are accepted).  Paged (vLLM flash
    layout): ``[num_pages, block_size, n_kv_heads, head_dim]`` with
    ``block_tables`` an int32 CUDA tensor ``[n_seqs, max_blocks]``.
    Contiguous: ``[n_rows, n_kv_heads, head_dim]``, sequence s occupying rows
    ``seq_row_offset[s] .. + seq_lens[s]`` (default: packed back to back).
    """
    k_layers: Sequence[torch.Tensor]
    v_layers: Sequence[torch.Tensor]
    seq_lens: Sequence[int]
    block_tables: Optional[torch.Tensor] = None
    seq_row_offset: Optional[Sequence[int]] = None
    layer_base: int = 0
    # split trees (dist.split_kv_commit): leaf position of each sequence's local
    # row 0, and a fixed subtree height (0: each tree padded to its own length)
    pos_base: Optional[Sequence[int]] = None
    tree_log2: int = 0


def _kv_desc(view: KvCacheView):
    if len(view.k_layers) == 0 or len(view.k_layers) != len(view.v_layers):
        raise ValueError("k_layers and v_layers must be non-empty and of equal length")
    k0 = view.k_layers[0]
    _require_cuda(k0, "k_layers[0]")
    if k0.dtype not in _DTYPES:
        raise ValueError(f"unsupported K/V dtype {k0.dtype}")
    paged = view.block_tables is not None
    for t in list(view.k_layers) + list(view.v_layers):
        _require_cuda(t, "K/V layer")
        if t.dtype != k0.dtype or t.shape != k0.shape:
            raise ValueError("all K/V layers must share one dtype and shape")
    d = KvDesc()
    d.n_layers = len(view.k_layers)
    d.layer_base = int(view.layer_base)
    d.dtype = _DTYPES[k0.dtype]
    d.n_seqs = len(view.seq_lens)
    keep = []
    if paged:
        if k0.dim() != 4:
            raise ValueError("paged K/V layers must be [num_pages, block_size, n_kv_heads, head_dim]")
        _require_cuda(view.block_tables, "block_tables")
        bt = view.block_tables
        if bt.dtype != torch.int32 or bt.dim() != 2 or not bt.is_contiguous():
            raise ValueError("block_tables must be a contiguous int32 [n_seqs, max_blocks] tensor")
        if bt.shape[0] < d.n_seqs:
            raise ValueError("block_tables has fewer rows than sequences")
        d.block_tables = bt.data_ptr()
        d.block_size = k0.shape[1]
        d.max_blocks_per_seq = bt.shape[1]
        d.n_kv_heads, d.head_dim = k0.shape[2], k0.shape[3]
        d.stride_page, d.stride_row, d.stride_head = k0.stride(0), k0.stride(1), k0.stride(2)
        if k0.stride(3) != 1:
            raise ValueError("head_dim must be contiguous")
    else:
        if k0.dim() != 3:
            raise ValueError("contiguous K/V layers must be [n_rows, n_kv_heads, head_dim]")
        d.block_tables = None
        d.block_size = 0
        d.max_blocks_per_seq = 0
        d.n_kv_heads, d.head_dim = k0.shape[1], k0.shape[2]
        d.stride_page, d.stride_row, d.stride_head = 0, k0.stride(0), k0.stride(1)
        if k0.stride(2) != 1:
            raise ValueError("head_dim must be contiguous")
    for t in list(view.k_layers) + list(view.v_layers):
        if t.stride() != k0.stride():
            raise ValueError("all K/V layers must share strides")
    # Elements reachable from the base pointer of each layer buffer.
    d.cache_elems = int(sum((s - 1) * st for s, st in zip(k0.shape, k0.stride())) + 1)
    seq_lens = _i32(view.seq_lens)
    keep.append(seq_lens)
    d.seq_lens = ctypes.cast(seq_lens, ctypes.POINTER(ctypes.c_int32))
    if view.seq_row_offset is not None:
        offs = _i64(view.seq_row_offset)
        keep.append(offs)
        d.seq_row_offset = ctypes.cast(offs, ctypes.POINTER(ctypes.c_int64))
    if view.pos_base is not None:
        pb = _i64(view.pos_base)
        keep.append(pb)
        d.pos_base = ctypes.cast(pb, ctypes.POINTER(ctypes.c_int64))
    d.tree_log2 = int(view.tree_log2)
    kp = _ptrs([t.data_ptr() for t in view.k_layers])
    vp = _ptrs([t.data_ptr() for t in view.v_layers])
    keep += [kp, vp]
    d.k_layers = ctypes.cast(kp, ctypes.POINTER(ctypes.c_void_p))
    d.v_layers = ctypes.cast(vp, ctypes.POINTER(ctypes.c_void_p))
    return d, keep


def kv_commit(ctx: Context, view: KvCacheView, keep_trees: bool = True,
              roots_out: Optional[torch.Tensor] = None):
    """Per-layer kv_roots of every sequence of ``view``.

    Returns ``(roots, trees)``: roots is a CUDA uint8 tensor
    ``[n_seqs, n_layers, 32]`` (sequence s's ``BatchCommitment.kv_roots``),
    trees a :class:`TreeSet` (tree ``s * n_layers + l``) or None.
    """
    d, keep = _kv_desc(view)
    if roots_out is None:
        roots_out = ctx.empty(d.n_seqs, d.n_layers, 32)
    if roots_out.numel() < d.n_seqs * d.n_layers * 32 or not roots_out.is_contiguous():
        raise ValueError("roots_out too small or not contiguous")
    h = ctypes.c_void_p()
    check(lib().vc_kv_commit(ctx.handle, ctypes.byref(d), ctypes.c_void_p(roots_out.data_ptr()),
                             ctypes.byref(h) if keep_trees else None))
    del keep
    return roots_out, (TreeSet(ctx, h) if keep_trees else None)


def kv_open(ctx: Context, view: KvCacheView, trees: TreeSet, seq: int, layers: Sequence[int],
            n_positions: int):
    """KV openings of open_v4 (prover/src/lib.rs:1564-1588) for one sequence.

    For each layer in ``layers`` and every position 0..n_positions-1: the
    ``KvEntry`` (K and V rows widened to f64) and its Merkle proof against
    that layer's kv_root.  Returns ``(entries f64 [n_sel, n_pos, 2, kv_dim],
    siblings uint8 [n_sel, n_pos, depth, 32], depth)``, all on the device.
    ``view`` and ``trees`` must be the ones the commit used, with the cache
    rows unchanged since.
    """
    d, keep = _kv_desc(view)
    kv = d.n_kv_heads * d.head_dim
    n_sel = len(layers)
    n = int(view.seq_lens[seq]) if 0 <= seq < len(view.seq_lens) else 1
    depth_max = max(1, (1 << (n - 1).bit_length()).bit_length() - 1) if n > 1 else 1
    depth_max = max(depth_max, int(view.tree_log2))
    entries = ctx.empty(max(n_sel, 1), max(n_positions, 1), 2, kv, dtype=torch.float64)
    sib = ctx.empty(max(n_sel, 1), max(n_positions, 1), depth_max, 32)
    depth = ctypes.c_int32(0)
    check(lib().vc_kv_open(ctx.handle, ctypes.byref(d), trees._h, int(seq), n_sel, _i32(layers), int(n_positions),
                           ctypes.c_void_p(entries.data_ptr()), ctypes.c_void_p(sib.data_ptr()), depth_max,
                           ctypes.byref(depth)))
    del keep
    return entries[:n_sel, :n_positions], sib[:n_sel, :n_positions, : depth.value], depth.value


class TreeGroups:
    """Tree sets of a KV commit done in layer groups; tree (s, l) lookups dispatch to the group."""

    def __init__(self, groups, n_seqs):
        self.groups = groups          # [(layer_begin, layer_end, TreeSet)]
        self.n_seqs = n_seqs

    def locate(self, seq: int, layer: int):
        for lb, le, ts in self.groups:
            if lb <= layer < le:
                return ts, seq * (le - lb) + (layer - lb)
        raise IndexError(f"layer {layer} not committed")

    def prove(self, seq: int, layer: int, positions: Sequence[int]):
        ts, t = self.locate(seq, layer)
        return ts.prove([t] * len(positions), positions)

    def free(self) -> None:
        for _, _, ts in self.groups:
            ts.free()


def kv_commit_host(ctx: Context, k_host: Sequence[torch.Tensor], v_host: Sequence[torch.Tensor],
                   seq_lens: Sequence[int], block_tables: Optional[torch.Tensor] = None,
                   seq_row_offset: Optional[Sequence[int]] = None, layer_base: int = 0, n_groups: int = 4,
                   dev_k: Optional[Sequence[torch.Tensor]] = None, dev_v: Optional[Sequence[torch.Tensor]] = None,
                   roots_out: Optional[torch.Tensor] = None, keep_trees: bool = True,
                   copy_stream: Optional[torch.cuda.Stream] = None):
    """kv_commit of a K/V transcript held in host memory (pinned for overlap).

    Layers are copied to the device in ``n_groups`` groups on a copy stream;
    each group is hashed on the context's stream as soon as its copy lands,
    while the next group is in flight.  ``dev_k``/``dev_v`` (same shapes on
    the device) are reused when given.  Returns ``(roots [n_seqs, n_layers,
    32], TreeGroups or None)``.
    """
    L = len(k_host)
    if L == 0 or L != len(v_host):
        raise ValueError("k_host and v_host must be non-empty and of equal length")
    dev = f"cuda:{ctx.device}"
    if dev_k is None:
        dev_k = [torch.empty_like(t, device=dev) for t in k_host]
    if dev_v is None:
        dev_v = [torch.empty_like(t, device=dev) for t in v_host]
    S = len(seq_lens)
    if roots_out is None:
        roots_out = ctx.empty(S, L, 32)
    cs = copy_stream if copy_stream is not None else torch.cuda.Stream(ctx.device)
    n_groups = max(1, min(n_groups, L))
    bounds = [L * i // n_groups for i in range(n_groups + 1)]
    groups = []
    for g in range(n_groups):
        lb, le = bounds[g], bounds[g + 1]
        # a device buffer is overwritten once the hashing that last read it is done:
        # each group's buffers carry the event of that launch (a buffer without one
        # waits for everything queued on the context so far)
        prior = {getattr(t, "_vc_read_done", None) for l in range(lb, le) for t in (dev_k[l], dev_v[l])}
        if None in prior:
            cs.wait_stream(ctx.stream)
        for ev_prev in prior - {None}:
            cs.wait_event(ev_prev)
        with torch.cuda.stream(cs):
            for l in range(lb, le):
                dev_k[l].copy_(k_host[l], non_blocking=True)
                dev_v[l].copy_(v_host[l], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(cs)
        ctx.stream.wait_event(ev)
        view = KvCacheView(dev_k[lb:le], dev_v[lb:le], seq_lens, block_tables=block_tables,
                           seq_row_offset=seq_row_offset, layer_base=layer_base + lb)
        if S == 1:
            out = roots_out[:, lb:le]
            r, ts = kv_commit(ctx, view, keep_trees=keep_trees, roots_out=out)
        else:
            r, ts = kv_commit(ctx, view, keep_trees=keep_trees, roots_out=ctx.empty(S, le - lb, 32))
            with torch.cuda.stream(ctx.stream):
                roots_out[:, lb:le].copy_(r.view(S, le - lb, 32))
        done = torch.cuda.Event()
        done.record(ctx.stream)
        for l in range(lb, le):
            dev_k[l]._vc_read_done = done
            dev_v[l]._vc_read_done = done
        if keep_trees:
            groups.append((lb, le, ts))
    return roots_out, (TreeGroups(groups, S) if keep_trees else None)


# ---------------------------------------------------------------------------
# Trees, IO chain, trace leaves
# ---------------------------------------------------------------------------

def build_trees(ctx: Context, leaves: torch.Tensor, leaf_off: Sequence[int], keep_trees: bool = True,
                roots_out: Optional[torch.Tensor] = None):
    """merkle::build_tree over each leaf range ``[leaf_off[i], leaf_off[i+1])`` of ``leaves [N, 32]``."""
    _require_cuda(leaves, "leaves")
    n_trees = len(leaf_off) - 1
    if roots_out is None:
        roots_out = ctx.empty(max(n_trees, 1), 32)
    h = ctypes.c_void_p()
    check(lib().vc_build_trees(ctx.handle, n_trees, _i64(leaf_off), ctypes.c_void_p(leaves.data_ptr()),
                               ctypes.c_void_p(roots_out.data_ptr()), ctypes.byref(h) if keep_trees else None))
    return roots_out[:n_trees], (TreeSet(ctx, h) if keep_trees else None)


def prompt_hashes(ctx: Context, prompts: Sequence[bytes]) -> torch.Tensor:
    """hash_prompt of each prompt, ``[n, 32]`` on the device."""
    off = [0]
    for p in prompts:
        off.append(off[-1] + len(p))
    data = ctx.to_device(b"".join(bytes(p) for p in prompts) or b"\0")
    out = ctx.empty(max(len(prompts), 1), 32)
    check(lib().vc_prompt_hash(ctx.handle, len(prompts), ctypes.c_void_p(data.data_ptr()), _i64(off),
                               ctypes.c_void_p(out.data_ptr())))
    return out[:len(prompts)]


def seed_commitments(ctx: Context, seeds: torch.Tensor) -> torch.Tensor:
    """hash_seed of each 32-byte seed (``[n, 32]`` uint8 CUDA tensor)."""
    _require_cuda(seeds, "seeds")
    n = seeds.shape[0]
    out = ctx.empty(max(n, 1), 32)
    check(lib().vc_seed_commitment(ctx.handle, n, ctypes.c_void_p(seeds.data_ptr()), ctypes.c_void_p(out.data_ptr())))
    return out[:n]


def io_chain(ctx: Context, leaves: torch.Tensor, token_ids: torch.Tensor, prompt_hash: torch.Tensor,
             tok_off: Sequence[int], out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """IO chain values of each sequence (tokens ``[tok_off[s], tok_off[s+1])``)."""
    for t, n in ((leaves, "leaves"), (token_ids, "token_ids"), (prompt_hash, "prompt_hash")):
        _require_cuda(t, n)
    if token_ids.dtype not in (torch.int32, torch.uint32):
        raise ValueError("token_ids must be a 32-bit CUDA tensor")
    if out is None:
        out = ctx.empty(max(leaves.shape[0], 1), 32)
    check(lib().vc_io_chain(ctx.handle, len(tok_off) - 1, _i64(tok_off), ctypes.c_void_p(leaves.data_ptr()),
                            ctypes.c_void_p(token_ids.data_ptr()), ctypes.c_void_p(prompt_hash.data_ptr()),
                            ctypes.c_void_p(out.data_ptr())))
    return out


@dataclass
class TraceLayout:
    """Per-token addressing of retained-state inputs already on the device.

    ``a_rows[f][l]`` / ``scale_a[f][l]``: device pointers (ints) of forward
    pass f, layer l; token t reads batch row ``tok_row[t]`` of pass
    ``tok_fwd[t]``.  Optional wraps: a CUDA tensor ``[rows, dim]`` plus a
    per-token row index list (-1: not bound).
    """
    n_layers: int
    hidden: int
    fwd_rows: Sequence[int]
    tok_fwd: Sequence[int]
    tok_row: Sequence[int]
    a_rows: Sequence[Sequence[int]]
    scale_a: Sequence[Sequence[int]]
    scale_stride: int = 1
    x_attn_rows: Optional[Sequence[Sequence[int]]] = None
    scale_x_attn: Optional[Sequence[Sequence[int]]] = None
    scale_x_stride: int = 1
    final_residual: Optional[torch.Tensor] = None
    tok_fr_row: Optional[Sequence[int]] = None
    lp_hidden: Optional[torch.Tensor] = None
    tok_lp_row: Optional[Sequence[int]] = None
    logits: Optional[torch.Tensor] = None
    tok_logits_row: Optional[Sequence[int]] = None


class TracePlan:
    """A ``vc_trace_desc`` built once from a :class:`TraceLayout`, for repeated commits."""

    def __init__(self, lay: TraceLayout):
        self.n = len(lay.tok_fwd)
        d = TraceDesc()
        keep = []
        d.n_tokens = self.n
        d.n_layers = lay.n_layers
        d.hidden = lay.hidden
        d.n_fwd = len(lay.fwd_rows)

        def arr32(x):
            a = np.ascontiguousarray(np.asarray(x, dtype=np.int32))
            keep.append(a)
            return a.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))

        def arrp(rows):
            a = np.ascontiguousarray(np.asarray(rows, dtype=np.uint64).reshape(-1))
            keep.append(a)
            return ctypes.cast(a.ctypes.data, ctypes.POINTER(ctypes.c_void_p))

        d.fwd_rows = arr32(lay.fwd_rows)
        d.tok_fwd = arr32(lay.tok_fwd)
        d.tok_row = arr32(lay.tok_row)
        d.a_rows = arrp(lay.a_rows)
        d.scale_a = arrp(lay.scale_a)
        d.scale_stride = int(lay.scale_stride)
        if lay.x_attn_rows is not None:
            d.x_attn_rows = arrp(lay.x_attn_rows)
            d.scale_x_attn = arrp(lay.scale_x_attn)
            d.scale_x_stride = int(lay.scale_x_stride)
        for name, ten, rows, esz in (("fr", lay.final_residual, lay.tok_fr_row, 4),
                                     ("lp", lay.lp_hidden, lay.tok_lp_row, 2),
                                     ("logits", lay.logits, lay.tok_logits_row, 4)):
            if ten is None:
                continue
            _require_cuda(ten, name)
            if ten.element_size() != esz or ten.dim() != 2 or ten.stride(1) != 1:
                raise ValueError(f"{name} must be a 2-D row-major tensor of {esz}-byte elements")
            ptr, dim, nrows, stride = ten.data_ptr(), ten.shape[1], ten.shape[0], ten.stride(0)
            if name == "fr":
                d.final_residual, d.fr_dim, d.fr_rows, d.fr_stride, d.tok_fr_row = ptr, dim, nrows, stride, arr32(rows)
            elif name == "lp":
                d.lp_hidden, d.lp_dim, d.lp_rows, d.lp_stride, d.tok_lp_row = ptr, dim, nrows, stride, arr32(rows)
            else:
                d.logits, d.vocab, d.logits_rows, d.logits_stride, d.tok_logits_row = ptr, dim, nrows, stride, arr32(rows)
        self.desc = d
        self._keep = keep

    def run(self, ctx: Context, out: torch.Tensor) -> torch.Tensor:
        if out.shape[0] < self.n or not out.is_contiguous():
            raise ValueError("out must be a contiguous [n_tokens, 32] uint8 CUDA tensor")
        check(lib().vc_trace_leaves(ctx.handle, ctypes.byref(self.desc), ctypes.c_void_p(out.data_ptr())))
        return out[: self.n]


def trace_leaves(ctx: Context, lay: TraceLayout, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Retained-state leaves of every token, ``[n_tokens, 32]`` on the device."""
    plan = TracePlan(lay)
    if out is None:
        out = ctx.empty(max(plan.n, 1), 32)
    return plan.run(ctx, out)


def int_peak(ctx: Context, variant: int = 0, iters: int = 20000) -> float:
    """Device-timed integer ops/s of the ALU probe (variant 0: SHA-256 mix)."""
    v = ctypes.c_double()
    check(lib().vc_int_peak(ctx.handle, int(variant), int(iters), ctypes.byref(v)))
    return v.value


def wait_probe(ctx: Context, limit_ns: int) -> None:
    """Queue the bounded-wait probe (``vc_wait_probe``): a wait that nothing
    satisfies gives up after ``limit_ns`` and flags the context, so the next
    :meth:`Context.sync` raises the timeout and the context stays usable."""
    check(lib().vc_wait_probe(ctx.handle, int(limit_ns)))


# --------------------------------------------------------------------------
# KV transcript: compute_kv_transcript (crates/verilm-prover/src/lib.rs:207-329)
# --------------------------------------------------------------------------

@dataclass
class RopeConfig:
    """RoPE part of ``ModelConfig`` (crates/verilm-core/src/constants.rs:126-156):
    ``theta`` and the optional scaling (``"llama3"``, ``"linear"``; any other
    type leaves the frequencies unscaled, constants.rs:292-295)."""
    theta: float = 10000.0
    scaling: Optional[str] = None
    factor: float = 8.0
    low_freq_factor: float = 1.0
    high_freq_factor: float = 4.0
    original_max_position_embeddings: int = 8192


@dataclass
class KvTranscriptInputs:
    """Device-resident inputs of one transcript.

    x_attn: per layer an int8 ``[n_tokens, hidden]`` view (row stride a
    multiple of 16 bytes, the same for every layer) or one
    ``[n_layers, n_tokens, hidden]`` tensor; wk, wv: per layer int8
    ``[kv_dim, hidden]`` row-major; scale_x: float32 ``[n_tokens, n_layers]``
    (any strides).  per_tensor: per layer ``(sw_k, sw_v)``; per_channel: per
    layer ``(cw_k, cw_v)`` float32 device tensors or None; biases: per layer
    ``(b_k, b_v)`` float32 device tensors or None.  With neither scale list
    the reference's toy path applies (clamp to int8).
    """
    x_attn: object
    wk: Sequence[torch.Tensor]
    wv: Sequence[torch.Tensor]
    scale_x: Optional[torch.Tensor]
    n_kv_heads: int
    head_dim: int
    per_tensor: Optional[Sequence] = None
    per_channel: Optional[Sequence] = None
    biases: Optional[Sequence] = None
    rope: Optional[RopeConfig] = None


def _kvt_desc(inp: KvTranscriptInputs):
    """(vc_kvt_desc, arrays it points to, n_layers, n_tokens, kv_dim) of the inputs."""
    xs = list(inp.x_attn) if not isinstance(inp.x_attn, torch.Tensor) else [x for x in inp.x_attn]
    n_layers = len(xs)
    if n_layers < 1 or len(inp.wk) != n_layers or len(inp.wv) != n_layers:
        raise ValueError("x_attn, wk and wv must have one entry per layer")
    n_tok, hidden = int(xs[0].shape[0]), int(xs[0].shape[1])
    stride = int(xs[0].stride(0))
    for x in xs:
        _require_cuda(x, "x_attn")
        if x.dtype != torch.int8 or tuple(x.shape) != (n_tok, hidden) or x.stride(1) != 1 or x.stride(0) != stride:
            raise ValueError("x_attn layers must be int8 [n_tokens, hidden] views with one common row stride")
    kv = int(inp.n_kv_heads) * int(inp.head_dim)
    for w in list(inp.wk) + list(inp.wv):
        _require_cuda(w, "weight")
        if w.dtype != torch.int8 or tuple(w.shape) != (kv, hidden) or not w.is_contiguous():
            raise ValueError(f"Wk/Wv must be contiguous int8 [{kv}, {hidden}]")
    use_rope = bool(inp.per_tensor) or bool(inp.per_channel)
    keep = []

    def pp(arr):
        keep.append(arr)
        return ctypes.cast(arr, ctypes.POINTER(ctypes.c_void_p))

    d = _lib.KvtDesc()
    d.n_tokens, d.n_layers, d.hidden = n_tok, n_layers, hidden
    d.n_kv_heads, d.head_dim, d.use_rope = int(inp.n_kv_heads), int(inp.head_dim), int(use_rope)
    d.x_layers = pp(_ptrs([x.data_ptr() for x in xs]))
    d.x_row_stride = stride
    d.wk_layers = pp(_ptrs([w.data_ptr() for w in inp.wk]))
    d.wv_layers = pp(_ptrs([w.data_ptr() for w in inp.wv]))
    if use_rope and n_tok > 0:
        sx = inp.scale_x
        _require_cuda(sx, "scale_x")
        if sx.dtype != torch.float32 or tuple(sx.shape) != (n_tok, n_layers):
            raise ValueError("scale_x must be float32 [n_tokens, n_layers]")
        d.scale_x, d.sx_tstride, d.sx_lstride = sx.data_ptr(), sx.stride(0), sx.stride(1)

        def per_layer(seq, m):
            out = []
            for l in range(n_layers):
                e = seq[l] if seq is not None and l < len(seq) and seq[l] is not None else None
                t = e[m] if e is not None else None
                if t is not None and t.numel() > 0:
                    _require_cuda(t, "scale/bias")
                    if t.dtype != torch.float32 or t.numel() != kv or not t.is_contiguous():
                        raise ValueError(f"per-channel scales and biases must be contiguous float32 [{kv}]")
                    out.append(t.data_ptr())
                else:
                    out.append(None)
            return pp(_ptrs(out))

        swk = (ctypes.c_float * n_layers)()
        swv = (ctypes.c_float * n_layers)()
        for l in range(n_layers):
            if inp.per_tensor and l < len(inp.per_tensor) and inp.per_tensor[l] is not None:
                swk[l], swv[l] = float(inp.per_tensor[l][0]), float(inp.per_tensor[l][1])
        d.sw_k = ctypes.cast(swk, ctypes.POINTER(ctypes.c_float))
        d.sw_v = ctypes.cast(swv, ctypes.POINTER(ctypes.c_float))
        d.ch_k, d.ch_v = per_layer(inp.per_channel, 0), per_layer(inp.per_channel, 1)
        d.bias_k, d.bias_v = per_layer(inp.biases, 0), per_layer(inp.biases, 1)
        keep += [swk, swv]
        r = inp.rope or RopeConfig()
        d.rope_theta = float(r.theta)
        d.rope_scaling = {"llama3": _lib.VC_ROPE_LLAMA3, "linear": _lib.VC_ROPE_LINEAR}.get(r.scaling or "",
                                                                                          _lib.VC_ROPE_NONE)
        d.rope_original_max_position_embeddings = int(r.original_max_position_embeddings)
        d.rope_factor, d.rope_low_freq_factor = float(r.factor), float(r.low_freq_factor)
        d.rope_high_freq_factor = float(r.high_freq_factor)
    return d, keep, n_layers, n_tok, kv


def kv_transcript(ctx: Context, inp: KvTranscriptInputs, k_out: Optional[torch.Tensor] = None,
                  v_out: Optional[torch.Tensor] = None):
    """``k_roped, v_deq``: float64 ``[n_layers, n_tokens, kv_dim]`` device tensors."""
    d, keep, n_layers, n_tok, kv = _kvt_desc(inp)
    if k_out is None:
        k_out = ctx.empty(n_layers, n_tok, kv, dtype=torch.float64)
    if v_out is None:
        v_out = ctx.empty(n_layers, n_tok, kv, dtype=torch.float64)
    for o in (k_out, v_out):
        if o.dtype != torch.float64 or tuple(o.shape) != (n_layers, n_tok, kv) or not o.is_contiguous():
            raise ValueError("outputs must be contiguous float64 [n_layers, n_tokens, kv_dim]")
    check(lib().vc_kv_transcript(ctx.handle, ctypes.byref(d), ctypes.c_void_p(k_out.data_ptr()),
                                 ctypes.c_void_p(v_out.data_ptr())))
    return k_out, v_out


def kv_transcript_commit(ctx: Context, inp: KvTranscriptInputs, layer_base: int = 0, keep_trees: bool = True,
                         roots_out: Optional[torch.Tensor] = None):
    """The per-layer kv_roots of the transcript of ``inp`` (positions 0..n_tokens-1,
    leaf layer index ``layer_base + l``), with the K/V rows hashed as they are
    computed and never stored: the roots and trees of :func:`kv_transcript`
    followed by :func:`kv_commit` of its rows.  Returns ``(roots [n_layers,
    32], TreeSet or None)`` (tree index = layer)."""
    d, keep, n_layers, n_tok, kv = _kvt_desc(inp)
    if roots_out is None:
        roots_out = ctx.empty(n_layers, 32)
    if roots_out.numel() < n_layers * 32 or not roots_out.is_contiguous():
        raise ValueError("roots_out too small or not contiguous")
    h = ctypes.c_void_p()
    check(lib().vc_kv_transcript_commit(ctx.handle, ctypes.byref(d), int(layer_base),
                                        ctypes.c_void_p(roots_out.data_ptr()),
                                        ctypes.byref(h) if keep_trees else None))
    del keep
    return roots_out.view(n_layers, 32), (TreeSet(ctx, h) if keep_trees else None)


def kv_transcript_view(k: torch.Tensor, v: torch.Tensor, layer_base: int = 0) -> KvCacheView:
    """The committed transcript as a one-sequence contiguous KV view (f64
    rows) for :func:`kv_commit` and :func:`kv_open`."""
    n_layers, n_tok, kv = k.shape
    return KvCacheView(k_layers=[k[l].view(n_tok, 1, kv) for l in range(n_layers)],
                       v_layers=[v[l].view(n_tok, 1, kv) for l in range(n_layers)],
                       seq_lens=[n_tok], layer_base=layer_base)
