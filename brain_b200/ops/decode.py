"""Paged-KV decode attention and the fused RoPE + KV-append of the new token (``csrc/attention_decode.cu``).

``paged_decode_attention(q, k_pool, v_pool, block_table, seq_lens)``: q [B, Hq, D] (one new token
per sequence, any strides with unit stride on D), pools [num_blocks, block_size, Hkv, D],
block_table [B, max_blocks] int32, seq_lens [B] int32 (cached tokens, the new one included).
The splits of a sequence merge inside one thread-block cluster, so no workspace is needed. With
programmatic dependent launch on (``set_pdl``), K/V older than the newest token are read before the
kernel waits on the preceding launch: a launch that may still run then must not write K/V below
position seq_lens[b] - 1 (the decode step writes only the newest token). On CPU the cache is gathered
per sequence and the reference SDPA is used. On the GPU the pool block size must be a multiple of 16
(K/V rows arrive as TMA boxes of 16 tokens).
"""
from __future__ import annotations

import math

import torch

from .. import _native
from ._common import same_device, stream

_native.register({
    "brain_decode_splits": ("brain_kernels", "iiii"),
    "brain_decode_attention": ("brain_kernels", "pllppipipiplliiiifippls"),
    "brain_kv_append_rope": ("brain_kernels", "pliiiipppppiis"),
    "brain_status_attention_decode": ("brain_kernels", "pi"),
})


def decode_splits(B: int, Hkv: int, D: int, max_len: int) -> int:
    """Split count (cluster size) of the decode attention for this batch shape on the current GPU."""
    return int(_native.fn("brain_decode_splits")(B, Hkv, D, max_len))


def paged_decode_attention(q, k_pool, v_pool, block_table, seq_lens, scale=None, splits=None, max_len=None,
                           out=None, trace=None, l2_prefetch=None):
    """``trace``: optional int64 CUDA tensor of (B * Hkv * splits * 8) elements that receives per-CTA
    globaltimer stamps (start, length read, after the wait, Q loaded, first chunk, loop end, cluster
    barrier, end) for profiling. ``l2_prefetch``: optional CUDA tensor (contiguous) that the CTAs ask
    L2 to load once their K/V stream is done, e.g. the weights of the kernel that follows."""
    B, Hq, D = q.shape
    Hkv = k_pool.shape[2]
    scale = scale if scale is not None else 1.0 / math.sqrt(D)
    same_device(q, k_pool, v_pool, block_table, seq_lens, out)
    if not q.is_cuda:
        return _decode_ref(q, k_pool, v_pool, block_table, seq_lens, scale)
    if splits is None:
        ml = max_len if max_len is not None else block_table.shape[1] * k_pool.shape[1]
        splits = decode_splits(B, Hkv, D, ml)
    if out is None:
        out = torch.empty(B, Hq, D, device=q.device, dtype=q.dtype)
    if not (k_pool.is_contiguous() and v_pool.is_contiguous() and block_table.is_contiguous()):
        raise ValueError("paged_decode_attention: K/V pools and the block table must be contiguous")
    _native.call("brain_decode_attention", q.data_ptr(), q.stride(0), q.stride(1), k_pool.data_ptr(),
                 v_pool.data_ptr(), k_pool.shape[0], block_table.data_ptr(), block_table.shape[1],
                 seq_lens.data_ptr(), k_pool.shape[1],
                 out.data_ptr(), out.stride(0), out.stride(1), B, Hq, Hkv, D, float(scale),
                 int(splits), trace.data_ptr() if trace is not None else 0,
                 l2_prefetch.data_ptr() if l2_prefetch is not None else 0,
                 l2_prefetch.numel() * l2_prefetch.element_size() if l2_prefetch is not None else 0, stream(q))
    return out


def _decode_ref(q, k_pool, v_pool, block_table, seq_lens, scale):
    B, Hq, D = q.shape
    Hkv = k_pool.shape[2]
    bs = k_pool.shape[1]
    out = torch.empty_like(q)
    for b in range(B):
        L = int(seq_lens[b])
        nb = -(-L // bs)
        idx = block_table[b, :nb].long()
        k = k_pool[idx].reshape(-1, Hkv, D)[:L].float()
        v = v_pool[idx].reshape(-1, Hkv, D)[:L].float()
        rep = Hq // Hkv
        kk, vv = k.repeat_interleave(rep, 1), v.repeat_interleave(rep, 1)  # [L, Hq, D]
        s = torch.einsum("hd,lhd->hl", q[b].float(), kk) * scale
        p = s.softmax(-1)
        out[b] = torch.einsum("hl,lhd->hd", p, vv).to(q.dtype)
    return out


def kv_append_rope(qkv, Hq, Hkv, pos, rope_cs, k_pool, v_pool, block_table):
    """qkv [B, (Hq+2Hkv)*D] of the new tokens: q and k rotated in place at positions pos [B] (int32),
    k and v written into the paged pools."""
    B = qkv.shape[0]
    D = qkv.shape[1] // (Hq + 2 * Hkv)
    if qkv.is_cuda:
        _native.call("brain_kv_append_rope", qkv.data_ptr(), qkv.stride(0), B, Hq, Hkv, D, pos.data_ptr(),
                     rope_cs.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(), block_table.data_ptr(),
                     block_table.shape[1], k_pool.shape[1], stream(qkv))
        return
    from .rope import rope_ref
    x = qkv.view(B, 1, Hq + 2 * Hkv, D)
    rot = rope_ref(x[:, :, :Hq + Hkv], rope_cs, pos.long()[:, None])
    x[:, :, :Hq + Hkv] = rot
    bs = k_pool.shape[1]
    for b in range(B):
        p = int(pos[b])
        blk = int(block_table[b, p // bs])
        k_pool[blk, p % bs] = x[b, 0, Hq:Hq + Hkv]
        v_pool[blk, p % bs] = x[b, 0, Hq + Hkv:]


# ---------------------------------------------------------------------------------------------
# Skinny (decode) GEMM with fused epilogues and the tensor-parallel step kernels (csrc/decode_tp.cu)
# ---------------------------------------------------------------------------------------------
EPI_STORE, EPI_PUSH, EPI_SWIGLU, EPI_QKV, EPI_ARGMAX = 0, 2, 3, 4, 5

_native.register({
    "brain_skinny_splits": ("brain_kernels", "iii"),
    "brain_skinny_gemm": ("brain_kernels", "plpliiiifplplips"),
    "brain_decode_set_pdl": ("brain_kernels", "i"),
    "brain_tp_ar_norm": ("brain_kernels", "ppiliiplpfplls"),
    "brain_tp_pick_embed": ("brain_kernels", "ppilipliippfpplppls"),
    "brain_status_decode_tp": ("brain_kernels", "pi"),
})


def set_pdl(mode) -> int:
    """Programmatic dependent launch for the decode-step kernels: 0/False off; 1/True on, a kernel's
    successor may launch as soon as it starts; 2 on, the skinny GEMM and the decode attention let their
    successor launch only after their main loop. Returns the previous mode."""
    return int(_native.fn("brain_decode_set_pdl")(int(mode)))


def skinny_splits(M: int, N: int, K: int) -> int:
    return int(_native.fn("brain_skinny_splits")(M, N, K))


def decode_ext(world=1, rank=0, slot_elems=0, ctrl=None, keys=None, vocab_offset=0, hq=0, hkv=0, pos=None,
               rope_cs=None, k_pool=None, v_pool=None, block_table=None, peer_slots=(), trace=None, l2_prefetch=None):
    """The int64[32] side-argument block of ``brain_skinny_gemm`` (layout documented in the source).
    ``l2_prefetch``: optional contiguous CUDA tensor that the CTAs ask L2 to load once their weights
    are consumed (the weights of a kernel that follows)."""
    import ctypes

    def p(t):
        return 0 if t is None else (t if isinstance(t, int) else t.data_ptr())
    v = [0] * 32
    v[0], v[1], v[2], v[3], v[4], v[5] = world, rank, slot_elems, p(ctrl), p(keys), vocab_offset
    v[6], v[7], v[8], v[9], v[10], v[11] = hq, hkv, p(pos), p(rope_cs), p(k_pool), p(v_pool)
    v[12], v[15] = p(block_table), p(trace)
    if block_table is not None:
        v[13], v[14] = block_table.shape[1], k_pool.shape[1]
    for i, s in enumerate(peer_slots):
        v[16 + i] = int(s)
    if l2_prefetch is not None:
        v[24], v[25] = l2_prefetch.data_ptr(), l2_prefetch.numel() * l2_prefetch.element_size()
    return (ctypes.c_int64 * 32)(*v)


def skinny_gemm(x, w, epi=EPI_STORE, out=None, residual=None, alpha=1.0, splits=None, ext=None, out_cols=None):
    """x [M, K] (M <= 64) times w [N, K]^T on the tensor cores with the operands swapped.

    epi: EPI_STORE (out [M, N], + residual), EPI_SWIGLU (w rows interleaved [gate 64 | up 64] per 128;
    out [M, N/2]), EPI_QKV / EPI_PUSH / EPI_ARGMAX (side arguments in ``ext``, see ``decode_ext``).
    """
    M, K = x.shape
    N = w.shape[0]
    same_device(x, w, out, residual)
    if splits is None:
        splits = skinny_splits(M, N, K)
    if out is None and epi in (EPI_STORE, EPI_SWIGLU, EPI_QKV):
        cols = out_cols if out_cols is not None else (N // 2 if epi == EPI_SWIGLU else N)
        out = torch.empty(M, cols, device=x.device, dtype=torch.bfloat16)
    _native.call("brain_skinny_gemm", x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), M, N, K, epi,
                 float(alpha), 0 if out is None else out.data_ptr(), 0 if out is None else out.stride(0),
                 0 if residual is None else residual.data_ptr(), 0 if residual is None else residual.stride(0),
                 int(splits), ext, stream(x))
    return out


def interleave_gate_up(w_gate, w_up, group: int = 64):
    """[F, K] gate and up weights -> [2F, K] with rows [gate 64 | up 64] per 128 (EPI_SWIGLU layout)."""
    F, K = w_gate.shape
    return torch.stack([w_gate.view(F // group, group, K), w_up.view(F // group, group, K)], 1).reshape(2 * F, K)


AR_SENTINEL = -0.0  # bf16 value marking an all-reduce receive slot element as not yet written


def init_ar_slots(slots: torch.Tensor) -> torch.Tensor:
    """Fill bf16 all-reduce receive slots with the sentinel (argmax key slots start at 0)."""
    return slots.view(torch.int16).fill_(-32768)


def ar_norm(slots, ctrl, world, slot_elems, resid, gamma, eps, normed, budget_s=2.0):
    """resid += sum of the `world` slots of the current epoch (polled until written, then reset to the
    sentinel); normed = rmsnorm(resid) * gamma."""
    M, N = resid.shape
    _native.call("brain_tp_ar_norm", slots, ctrl.data_ptr(), world, slot_elems, M, N, resid.data_ptr(),
                 resid.stride(0), gamma.data_ptr(), float(eps), normed.data_ptr(), normed.stride(0),
                 int(budget_s * 1e9), stream(resid))


def pick_embed(key_slots, ctrl, world, slot_elems, emb, resid, gamma, eps, normed, hist, pos, seq_lens, budget_s=2.0):
    """Greedy token from the ranks' argmax keys -> hist / pos / seq_lens, and the next layer-0 input."""
    M, N = resid.shape
    _native.call("brain_tp_pick_embed", key_slots, ctrl.data_ptr(), world, slot_elems, M, emb.data_ptr(),
                 emb.stride(0), emb.shape[0], N, resid.data_ptr(), gamma.data_ptr(), float(eps), normed.data_ptr(),
                 hist.data_ptr(), hist.stride(0), pos.data_ptr(), seq_lens.data_ptr(), int(budget_s * 1e9),
                 stream(resid))
