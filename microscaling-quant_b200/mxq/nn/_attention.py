"""The attention core through two Schemes (mxq/nn/_attention.py:70-167): S = Q·Kᵀ through `qk`, scale, additive
mask and softmax in float32 (or each step rounded to bf16), O = P·V through `pv`.

    o = attend(q, k, v, mask, scale, qk, pv, chunk=None, vector=None)   q: B×H×Tq×D, k, v: B×Hkv×Tk×D, o: B×Tq×H×D

Per batch row and KV head, with the group's query heads side by side as the columns of one call (head-major):
Kᵀ and V are quantized once per KV head, blocks along their contraction (D for Q·Kᵀ, the keys for P·V); each query
chunk's Qᵀ and Pᵀ once. Chunks are whole multiples of the Schemes' `rows` (a LUT table never straddles two heads);
the tokens left over run one head at a time.

Masked keys (mxq/nn/_attention.py:24-37, :117-141): the key blocks that a chunk's mask removes for every one of its
queries are not computed. A removed key's score would be fl(fl(S·scale) + mask), which is the mask value itself
when |S·scale| is below half an ulp of it; `_live_keys` keeps every key where that is not certain, from a bound on
|S·scale| taken from the quantized operands (Σ_d max|Q̂_d|·max|K̂_d| · |scale| · 2^16 for the reducer's roundings),
checked against the mask values in float32. A causal or padding mask at dtype-min passes; a -1e4 mask or a stray
finite value computes every key. The skipped scores are filled with the mask values (rounded like a computed one
under vector="bf16"), softmax runs on whole rows, and P·V contracts over the kept key blocks only when P is exactly
zero at the skipped keys (zero codes add zero tiles, which every reducer's tile add leaves unchanged); a query row
whose keys are all removed has a uniform P, and then every key block is contracted. The bits are those of computing
every key.

When both Schemes are this package's block quantizers (along axis 0) and systolic reducer, with rows = 1, all the
batch rows and heads go through at once instead (`_attend_stacked`): every Kᵀ, V, Qᵀ and Pᵀ of a pass quantized in
one call (a stack of matrices, blocks along each matrix's contraction) and every product in one batched systolic
launch. The operations per matrix are the same, so are the bits; only the number of launches changes. With a mask
the stacked path runs the queries in chunks (`chunk`, else a quarter of Tq in whole `rows`) and skips each chunk's
removed key blocks over the pass's batch rows together: for a causal mask that is 5/8 of the keys' work.

Registered as transformers' attention implementation "mxq" (`register`), which patch() switches a model to.
"""
from functools import partial
from typing import Optional

import torch

from ..block import BLOCK
from ..scheme import Scheme
from ._vector import rounder, softmax

__all__ = ["attend", "register", "NAME"]

NAME = "mxq"
#: score entries (n·m × Tk) per call when `chunk` is None
ELEMENTS_PER_STEP = 1 << 26
#: how far a reducer's score can exceed the exact sum of its absolute products through its roundings: under a
#: factor (1 + 2^-(m+1)) per rounding, below 2^16 for any lane width over 32 roundings and 256 block adds
SLACK = 2.0 ** 16
#: query chunks per stacked pass when a mask is given and `chunk` is None
MASKED_CHUNKS = 4


def _row_amax(P: torch.Tensor, X: torch.Tensor, block_size: int) -> torch.Tensor:
    """Largest dequantized magnitude of each contraction row of codes P (... × K × n) with scales X
    (... × ceil(K / block) × n), as float64 (... × K)."""
    K = P.shape[-2]
    return (P.abs() * X.repeat_interleave(block_size, dim=-2)[..., :K, :]).amax(dim=-1).double()


def _live_keys(mask_rows: torch.Tensor, bound: float, Tk: int, bv: int):
    """[lo, hi): the key blocks (of bv keys) holding every key some query of `mask_rows` (... × Tk, float32) may
    still see, given |S·scale| <= bound; a key is dead only where mask + bound and mask - bound both round back to
    the mask value. (0, bv) when every key is dead."""
    m = mask_rows.reshape(-1, Tk)
    dead = ((m + bound) == m) & ((m - bound) == m)
    live = (~dead.all(dim=0)).nonzero()
    if live.numel() == 0:
        return 0, min(Tk, bv)
    first, last = int(live[0]), int(live[-1])
    return first // bv * bv, min(Tk, -(-(last + 1) // bv) * bv)


def _stacked(s: Scheme):
    """(a, b, reduce) applying the Scheme to a stack of matrices (S×K×M), one call each, when its quantizers are
    this package's block quantizers along axis 0 and its reducer is systolic; else None."""
    from .. import block
    from ..matmul import _systolic
    if s.rows != 1:
        return None

    def quantizer(fn):
        if (not isinstance(fn, partial) or len(fn.args) > 1 or
                fn.func not in (block.mxquant.quantize, block.mxgemmini.quantize, block.ocp.quantize)):
            return None
        kw = dict(fn.keywords)
        if kw.get("axis", 0) != 0 or kw.get("block_size", BLOCK) != s.block_size:
            return None
        kw["axis"] = 1                                     # blocks along each matrix's rows, never across matrices
        return lambda V3: fn.func(V3, *fn.args, **kw)

    r = s.reduce
    if not isinstance(r, partial) or r.func is not _systolic.systolic or r.args:
        return None
    kw = dict(r.keywords)
    if kw.get("block_size", BLOCK) != s.block_size:
        return None
    a, b = quantizer(s.a), quantizer(s.b)
    if a is None or b is None:
        return None
    return a, b, lambda PA, XA, PB, XB: _systolic.systolic_batched(PA, XA, PB, XB, **kw)


def _attend_stacked(q, k, v, mask, scale, qk, pv, plan_qk, plan_pv, vector, chunk):
    """attend with every (batch row, KV head) of a pass stacked: the per-head loop's operations, batched. With a
    mask, the queries run in chunks and each chunk skips the key blocks its mask removes for all of the pass."""
    B, H, Tq, D = q.shape
    Hkv, Tk = k.shape[1], k.shape[2]
    group = H // Hkv
    rows = max(qk.rows, pv.rows)
    bq, bv = qk.block_size, pv.block_size
    r = rounder(vector)
    qa, qb, qred = plan_qk
    pa, pb, pred = plan_pv
    out = q.new_empty(B, Tq, H, D)
    if mask is None:
        step = Tq
    elif chunk:
        step = chunk
    else:
        quarter = -(-Tq // MASKED_CHUNKS)
        step = -(-quarter // rows) * rows                                       # whole rows
    per = max(1, (4 * ELEMENTS_PER_STEP) // max(1, H * min(step, Tq) * Tk))   # batch rows per pass
    tiny = torch.finfo(torch.float32).tiny
    for b0 in range(0, B, per):
        b1 = min(B, b0 + per)
        nb, n = b1 - b0, (b1 - b0) * Hkv
        KT = qb(k[b0:b1].float().transpose(-1, -2).reshape(n, D, Tk).contiguous())   # Kᵀ: D×Tk per KV head
        V = pb(v[b0:b1].float().reshape(n, Tk, D).contiguous())                      # V: Tk×D
        qk.check_scales(KT[1][0], D, "b (Kᵀ)")
        pv.check_scales(V[1][0], Tk, "b (V)")
        mb = None
        if mask is not None:
            mb = mask[b0:b1] if mask.shape[0] > 1 else mask[:1].expand(nb, *mask.shape[1:])
            mb = mb[:, 0, :, :Tk].float()
            mb = mb.expand(nb, Tq, Tk) if mb.shape[1] == 1 else mb
            kmax = _row_amax(*KT, bq).amax(dim=0)                                   # D: over every key of the pass
        for s0 in range(0, Tq, step):
            s1 = min(Tq, s0 + step)
            m = s1 - s0
            Q = q[b0:b1, :, s0:s1].float().reshape(n, group * m, D).transpose(1, 2).contiguous()  # D × group·m
            A = qa(Q)
            lo, hi = 0, Tk
            if mb is not None:
                qmax = _row_amax(*A, bq).amax(dim=0)
                bound = max(SLACK * abs(scale) * float((qmax * kmax).sum()), tiny)
                lo, hi = _live_keys(mb[:, s0:s1], bound, Tk, bv)
            if lo == 0 and hi == Tk:
                S = r(qred(*A, *KT) * scale)                                            # n × group·m × Tk
                if mb is not None:
                    S = r((S.view(nb, Hkv, group, m, Tk) + mb[:, None, None, s0:s1]).view(n, group * m, Tk))
            else:
                kt = (KT[0][:, :, lo:hi].contiguous(), KT[1][:, :, lo:hi].contiguous())
                live = r(qred(*A, *kt) * scale).view(nb, Hkv, group, m, hi - lo)
                S = r(mb[:, None, None, s0:s1]).expand(nb, Hkv, group, m, Tk).clone()   # removed keys: the mask
                S[..., lo:hi] = r(live + mb[:, None, None, s0:s1, lo:hi])
                S = S.view(n, group * m, Tk)
            P = softmax(S, vector)
            if (lo or hi < Tk) and (P[..., :lo].any() or P[..., hi:].any()):
                lo, hi = 0, Tk                                                          # a row with no live key
            PA = pa(P.transpose(1, 2).contiguous())                                     # Pᵀ: Tk × group·m
            if lo == 0 and hi == Tk:
                O = pred(*PA, *V)                                                        # group·m × D
            else:
                blk = slice(lo // bv, -(-hi // bv))
                O = pred(PA[0][:, lo:hi].contiguous(), PA[1][:, blk].contiguous(), V[0][:, lo:hi].contiguous(),
                         V[1][:, blk].contiguous())
            out[b0:b1, s0:s1] = O.view(nb, H, m, D).transpose(1, 2).to(q.dtype)
    return out


@torch.no_grad()
def attend(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask: Optional[torch.Tensor], scale: float,
           qk: Scheme, pv: Scheme, chunk: Optional[int] = None, vector: Optional[str] = None) -> torch.Tensor:
    """Attention with S = Q·Kᵀ through `qk` and O = P·V through `pv`; mask None or additive, broadcastable to
    B×1×Tq×Tk. chunk: query tokens per call, a positive multiple of the Schemes' rows."""
    B, H, Tq, D = q.shape
    Hkv, Tk = k.shape[1], k.shape[2]
    if H % Hkv or v.shape[1] != Hkv or v.shape[2] != Tk:
        raise ValueError(f"attend: q has {H} heads, k {tuple(k.shape)}, v {tuple(v.shape)}")
    rows = max(qk.rows, pv.rows)
    if chunk is not None and (chunk < 1 or chunk % rows):
        raise ValueError(f"attend: chunk {chunk} must be a positive multiple of the schemes' rows = {rows}")
    group = H // Hkv
    plan_qk, plan_pv = _stacked(qk), _stacked(pv)
    if plan_qk is not None and plan_pv is not None:
        return _attend_stacked(q, k, v, mask, scale, qk, pv, plan_qk, plan_pv, vector, chunk)
    step = chunk or max(rows, ELEMENTS_PER_STEP // (group * Tk) // rows * rows)
    bq, bv = qk.block_size, pv.block_size
    tiny = torch.finfo(torch.float32).tiny
    r = rounder(vector)
    out = q.new_empty(B, Tq, H, D)
    for b in range(B):
        mb = None
        if mask is not None:
            mb = mask[b if mask.shape[0] > 1 else 0, 0, :, :Tk].float()
            mb = mb.expand(Tq, Tk) if mb.shape[0] == 1 else mb
        for h in range(Hkv):
            KT = qk.b(k[b, h].float().t().contiguous())                     # Kᵀ: D×Tk, blocks along D
            V = pv.b(v[b, h].float().contiguous())                          # V: Tk×D, blocks along the keys
            qk.check_scales(KT[1], D, "b (Kᵀ)")
            pv.check_scales(V[1], Tk, "b (V)")
            kmax = _row_amax(*KT, bq) if mb is not None else None
            heads = range(h * group, (h + 1) * group)
            for s in range(0, Tq, step):
                e = min(s + step, Tq)
                whole = s + (e - s) // rows * rows                          # every head at once up to here
                parts = [(heads, s, whole)] if whole > s else []
                parts += [(range(hq, hq + 1), whole, e) for hq in heads] if whole < e else []
                for hs, s0, e0 in parts:
                    n, m = len(hs), e0 - s0
                    Q = q[b, hs.start:hs.stop, s0:e0].float().reshape(n * m, D)  # n·m×D, head-major
                    A = qk.a(Q.t().contiguous())
                    lo, hi = 0, Tk
                    if mb is not None:
                        bound = max(SLACK * abs(scale) * float((_row_amax(*A, bq) * kmax).sum()), tiny)
                        lo, hi = _live_keys(mb[s0:e0], bound, Tk, bv)
                    if lo == 0 and hi == Tk:
                        S = r(qk.reduce(*A, *KT) * scale)                     # n·m×Tk
                        if mb is not None:
                            S = r((S.view(n, m, Tk) + mb[s0:e0]).view(n * m, Tk))
                    else:
                        live = r(qk.reduce(*A, KT[0][:, lo:hi].contiguous(), KT[1][:, lo:hi].contiguous()) * scale)
                        S = r(mb[s0:e0]).repeat(n, 1)                         # removed keys: the mask values
                        S.view(n, m, Tk)[:, :, lo:hi] = r(live.view(n, m, hi - lo) + mb[s0:e0, lo:hi])
                    P = softmax(S, vector)
                    if (lo or hi < Tk) and (P[:, :lo].any() or P[:, hi:].any()):
                        lo, hi = 0, Tk                                        # a row with no live key: P uniform
                    PA = pv.a(P.t().contiguous())                             # Pᵀ: Tk×n·m, blocks along the keys
                    if lo == 0 and hi == Tk:
                        O = pv.reduce(*PA, *V)                                # n·m×D
                    else:
                        blk = slice(lo // bv, -(-hi // bv))
                        O = pv.reduce(PA[0][lo:hi].contiguous(), PA[1][blk].contiguous(), V[0][lo:hi].contiguous(),
                                      V[1][blk].contiguous())
                    out[b, s0:e0, hs.start:hs.stop] = O.view(n, m, D).transpose(0, 1).to(q.dtype)
    return out


def _mxq_attention(module, query, key, value, attention_mask, dropout: float = 0.0,
                   scaling: Optional[float] = None, **kwargs):
    """transformers' attention-function signature; a module patch() gave no core runs sdpa unchanged."""
    core = getattr(module, "_mxq_core", None)
    if core is None:
        from transformers.integrations.sdpa_attention import sdpa_attention_forward
        return sdpa_attention_forward(module, query, key, value, attention_mask, dropout=dropout, scaling=scaling,
                                      **kwargs)
    if dropout:
        raise ValueError("mxq attention is inference only: dropout must be 0")
    qk, pv = core
    scale = scaling if scaling is not None else query.shape[-1] ** -0.5
    return attend(query, key, value, attention_mask, scale, qk, pv, vector=getattr(module, "_mxq_vector", None)), None


def register() -> None:
    """Make NAME a transformers attention implementation with eager's additive float mask. Safe to repeat."""
    from transformers import AttentionInterface
    from transformers.masking_utils import AttentionMaskInterface, eager_mask
    AttentionInterface.register(NAME, _mxq_attention)
    AttentionMaskInterface.register(NAME, eager_mask)
