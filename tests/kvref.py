"""Build the same K/V transcript for the GPU path and for the oracle.

Test helper: the GPU side gets a ``KvCacheView`` over CUDA tensors, the
oracle side a ``vc_kv_desc`` over the very same host arrays.
"""
from __future__ import annotations

import ctypes

import numpy as np

from commitllm_b200._lib import KvDesc, VC_DTYPE_BF16, VC_DTYPE_F32, VC_DTYPE_F64
from oracle import vco

NP_DT = {VC_DTYPE_BF16: np.uint16, VC_DTYPE_F32: np.float32, VC_DTYPE_F64: np.float64}


class Transcript:
    """K/V layers as host arrays plus the addressing of one cache layout.

    ``k``/``v``: ``[n_layers, *buffer_shape]`` host arrays where a layer
    buffer is ``[pages, block, heads, dim]`` (paged) or ``[rows, heads, dim]``
    (contiguous), or an HND-style permutation given by ``strides``.
    """

    def __init__(self, k, v, seq_lens, dtype, block_tables=None, seq_row_offset=None, layer_base=0):
        self.k, self.v = np.ascontiguousarray(k), np.ascontiguousarray(v)
        self.seq_lens = [int(x) for x in seq_lens]
        self.dtype = dtype
        self.block_tables = None if block_tables is None else np.ascontiguousarray(block_tables, dtype=np.int32)
        self.seq_row_offset = seq_row_offset
        self.layer_base = layer_base

    # --- oracle side ---
    def oracle_desc(self, k=None, v=None):
        k = self.k if k is None else k
        v = self.v if v is None else v
        d = KvDesc()
        keep = [k, v]
        L = k.shape[0]
        d.n_layers = L
        d.layer_base = self.layer_base
        d.dtype = self.dtype
        d.n_seqs = len(self.seq_lens)
        es = k.itemsize
        st = [s // es for s in k.strides[1:]]
        if self.block_tables is not None:
            d.n_kv_heads, d.head_dim = k.shape[3], k.shape[4]
            d.block_size = k.shape[2]
            d.block_tables = self.block_tables.ctypes.data
            d.max_blocks_per_seq = self.block_tables.shape[1]
            d.stride_page, d.stride_row, d.stride_head = st[0], st[1], st[2]
            keep.append(self.block_tables)
        else:
            d.n_kv_heads, d.head_dim = k.shape[2], k.shape[3]
            d.stride_page, d.stride_row, d.stride_head = 0, st[0], st[1]
        d.cache_elems = k[0].size
        sl = (ctypes.c_int32 * len(self.seq_lens))(*self.seq_lens)
        keep.append(sl)
        d.seq_lens = ctypes.cast(sl, ctypes.POINTER(ctypes.c_int32))
        if self.seq_row_offset is not None:
            ro = (ctypes.c_int64 * len(self.seq_row_offset))(*self.seq_row_offset)
            keep.append(ro)
            d.seq_row_offset = ctypes.cast(ro, ctypes.POINTER(ctypes.c_int64))
        kp = (ctypes.c_void_p * L)(*[k[l].ctypes.data for l in range(L)])
        vp = (ctypes.c_void_p * L)(*[v[l].ctypes.data for l in range(L)])
        keep += [kp, vp]
        d.k_layers = ctypes.cast(kp, ctypes.POINTER(ctypes.c_void_p))
        d.v_layers = ctypes.cast(vp, ctypes.POINTER(ctypes.c_void_p))
        return d, keep

    def oracle(self, n_threads=8, with_nodes=True):
        """(roots [n_seqs, n_layers, 32], list of node arrays per tree or None)."""
        d, keep = self.oracle_desc()
        L, S = d.n_layers, d.n_seqs
        roots = np.zeros((S, L, 32), np.uint8)
        nodes = node_off = None
        offs = []
        if with_nodes:
            tot = 0
            for s in range(S):
                n = self.seq_lens[s]
                pad = 1 << (n - 1).bit_length() if n > 1 else 1
                for _l in range(L):
                    offs.append((tot, pad))
                    tot += 2 * pad - 1
            nodes = np.zeros((tot, 32), np.uint8)
            node_off = np.array([o for o, _ in offs], dtype=np.int64)
        rc = vco.lib().vco_kv_commit(ctypes.byref(d), roots.ctypes.data, None if nodes is None else nodes.ctypes.data,
                                     None if node_off is None else node_off.ctypes.data, n_threads)
        assert rc == 0
        del keep
        trees = [nodes[o:o + 2 * p - 1] for o, p in offs] if with_nodes else None
        return roots, trees

    # --- GPU side ---
    def view(self, device=0):
        import torch
        from commitllm_b200.commit import KvCacheView
        tdt = {VC_DTYPE_BF16: torch.int16, VC_DTYPE_F32: torch.float32, VC_DTYPE_F64: torch.float64}[self.dtype]

        def dev(a):
            t = torch.from_numpy(np.ascontiguousarray(a).view(NP_DT[self.dtype]).view(
                {VC_DTYPE_BF16: np.int16, VC_DTYPE_F32: np.float32, VC_DTYPE_F64: np.float64}[self.dtype]))
            return t.to(f"cuda:{device}")

        kd, vd = dev(self.k), dev(self.v)
        if self.k.strides != np.ascontiguousarray(self.k).strides:
            raise ValueError("host arrays must be C-contiguous")
        bt = None if self.block_tables is None else torch.from_numpy(self.block_tables).to(f"cuda:{device}")
        view = KvCacheView(k_layers=[kd[l] for l in range(kd.shape[0])], v_layers=[vd[l] for l in range(vd.shape[0])],
                           seq_lens=self.seq_lens, block_tables=bt, seq_row_offset=self.seq_row_offset,
                           layer_base=self.layer_base)
        view._keep = (kd, vd, bt)
        return view


def contiguous(seed, n_layers, seq_lens, n_heads, head_dim, dtype=VC_DTYPE_BF16, layer_base=0):
    rows = sum(seq_lens)
    rng = np.random.default_rng(seed)
    shape = (n_layers, rows, n_heads, head_dim)
    if dtype == VC_DTYPE_BF16:
        from tests.synth import f32_to_bf16_bits
        k = f32_to_bf16_bits(rng.standard_normal(shape, dtype=np.float32))
        v = f32_to_bf16_bits(rng.standard_normal(shape, dtype=np.float32))
    elif dtype == VC_DTYPE_F32:
        k = rng.standard_normal(shape, dtype=np.float32)
        v = rng.standard_normal(shape, dtype=np.float32)
    else:
        k = rng.standard_normal(shape)
        v = rng.standard_normal(shape)
    return Transcript(k, v, seq_lens, dtype, layer_base=layer_base)


def paged(seed, n_layers, seq_lens, n_heads, head_dim, block_size=16, extra_pages=3, dtype=VC_DTYPE_BF16):
    rng = np.random.default_rng(seed)
    need = [(n + block_size - 1) // block_size for n in seq_lens]
    n_pages = sum(need) + extra_pages
    perm = rng.permutation(n_pages).astype(np.int32)
    mb = max(need)
    bt = np.full((len(seq_lens), mb), -7, dtype=np.int32)   # unused slots hold junk
    c = 0
    for s, k in enumerate(need):
        bt[s, :k] = perm[c:c + k]
        c += k
    shape = (n_layers, n_pages, block_size, n_heads, head_dim)
    from tests.synth import f32_to_bf16_bits
    if dtype == VC_DTYPE_BF16:
        k = f32_to_bf16_bits(rng.standard_normal(shape, dtype=np.float32))
        v = f32_to_bf16_bits(rng.standard_normal(shape, dtype=np.float32))
    elif dtype == VC_DTYPE_F32:
        k = rng.standard_normal(shape, dtype=np.float32)
        v = rng.standard_normal(shape, dtype=np.float32)
    else:
        k = rng.standard_normal(shape)
        v = rng.standard_normal(shape)
    return Transcript(k, v, seq_lens, dtype, block_tables=bt)
