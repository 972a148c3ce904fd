"""The attention core through two Schemes (mxq/nn/_attention.py:70-167): S = Q·Kᵀ through `qk`, scale, additive
mask and softmax in float32 (or each step rounded to bf16), O = P·V through `pv`.

    o = attend(q, k, v, mask, scale, qk, pv, chunk=None, vector=None)   q: B×H×Tq×D, k, v: B×Hkv×Tk×D, o: B×Tq×H×D

Per batch row and KV head, with the group's query heads side by side as the columns of one call (head-major):
Kᵀ and V are quantized once per KV head, blocks along their contraction (D for Q·Kᵀ, the keys for P·V); each query
chunk's Qᵀ and Pᵀ once. Chunks are whole multiples of the Schemes' `rows` (a LUT table never straddles two heads);
the tokens left over run one head at a time. Every key is computed: the reference's skipping of key blocks the mask
removes for every query produces the same bits (the skipped scores equal the mask values and the skipped P·V blocks
add zero tiles), so here it is only a matter of speed.

When both Schemes are this package's block quantizers (along axis 0) and systolic reducer, with rows = 1, all the
batch rows and heads go through at once instead (`_attend_stacked`): every Kᵀ, V, Qᵀ and Pᵀ of a pass quantized in
one call (a stack of matrices, blocks along each matrix's contraction) and every product in one batched systolic
launch. The operations per matrix are the same, so are the bits; only the number of launches changes.

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


def _attend_stacked(q, k, v, mask, scale, qk, pv, plan_qk, plan_pv, vector):
    """attend with every (batch row, KV head) of a pass stacked: the per-head loop's operations, batched."""
    B, H, Tq, D = q.shape
    Hkv, Tk = k.shape[1], k.shape[2]
    group = H // Hkv
    r = rounder(vector)
    qa, qb, qred = plan_qk
    pa, pb, pred = plan_pv
    out = q.new_empty(B, Tq, H, D)
    per = max(1, (4 * ELEMENTS_PER_STEP) // max(1, H * Tq * Tk))          # batch rows per pass (scores in memory)
    for b0 in range(0, B, per):
        b1 = min(B, b0 + per)
        nb, n = b1 - b0, (b1 - b0) * Hkv
        KT = k[b0:b1].float().transpose(-1, -2).reshape(n, D, Tk).contiguous()      # Kᵀ: D×Tk per KV head
        V = v[b0:b1].float().reshape(n, Tk, D).contiguous()                         # V: Tk×D
        KT = qb(KT)
        V = pb(V)
        qk.check_scales(KT[1][0], D, "b (Kᵀ)")
        pv.check_scales(V[1][0], Tk, "b (V)")
        Q = q[b0:b1].float().reshape(n, group * Tq, D).transpose(1, 2).contiguous()  # Qᵀ: D × group·Tq, head-major
        A = qa(Q)
        S = r(qred(*A, *KT) * scale)                                                # n × group·Tq × Tk
        if mask is not None:
            mb = mask[b0:b1] if mask.shape[0] > 1 else mask[:1].expand(nb, *mask.shape[1:])
            mb = mb[:, 0, :, :Tk].float()
            mb = mb.expand(nb, Tq, Tk) if mb.shape[1] == 1 else mb
            S = r((S.view(nb, Hkv, group, Tq, Tk) + mb[:, None, None]).view(n, group * Tq, Tk))
        P = softmax(S, vector)
        PA = pa(P.transpose(1, 2).contiguous())                                     # Pᵀ: Tk × group·Tq
        O = pred(*PA, *V)                                                            # group·Tq × D
        out[b0:b1] = O.view(nb, H, Tq, D).transpose(1, 2).to(q.dtype)
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
        return _attend_stacked(q, k, v, mask, scale, qk, pv, plan_qk, plan_pv, vector)
    step = chunk or max(rows, ELEMENTS_PER_STEP // (group * Tk) // rows * rows)
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
                    S = r(qk.reduce(*A, *KT) * scale)                         # n·m×Tk
                    if mb is not None:
                        S = r((S.view(n, m, Tk) + mb[s0:e0]).view(n * m, Tk))
                    P = softmax(S, vector)
                    PA = pv.a(P.t().contiguous())                             # Pᵀ: Tk×n·m, blocks along the keys
                    O = pv.reduce(*PA, *V)                                    # n·m×D
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
