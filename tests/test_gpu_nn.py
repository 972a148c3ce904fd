"""mxq.nn on the GPU against the reference: MXLinear and Scheme.matmul bit for bit; attend within the float32
softmax's tolerance (torch's softmax sums in another order on the GPU, so a probability can move by an ulp; the
north-star tolerance for the glue is 1e-6 relative); and a config-5-style patched Llama, where every MXLinear run
on the reference's own captured input must give the reference's output bit for bit and the logits agree to the
glue tolerance."""
from functools import partial

import numpy as np
import pytest
import torch

from _util import assert_bits, golden

pytestmark = pytest.mark.gpu


def hw_scheme():
    import mxq
    from mxq import Scheme, block, matmul, schedule
    q = partial(block.mxgemmini.quantize, fmt="MXFP8_E4M3", axis=0)
    return Scheme("hw_fp8", a=q, b=q, reduce=partial(matmul.systolic, arith=matmul.MXGEMMINI(),
                                                      schedule=schedule.HW_FINAL))


def test_mxlinear_golden():
    from mxq.nn import MXLinear
    g = golden("nn")
    lin = torch.nn.Linear(96, 40, bias=True)
    with torch.no_grad():
        lin.weight.copy_(torch.from_numpy(g["linear/W"]))
        lin.bias.copy_(torch.from_numpy(g["linear/b"]))
    lin = lin.cuda()
    x = torch.from_numpy(g["linear/x"]).cuda()
    assert_bits(MXLinear(lin, hw_scheme())(x), g["linear/y"], "MXLinear")
    assert_bits(MXLinear(lin, hw_scheme(), chunk=5)(x), g["linear/y_chunk5"], "MXLinear chunk 5")


def test_scheme_golden():
    g = golden("nn")
    Y = hw_scheme().matmul(torch.from_numpy(g["scheme/A"]).cuda(), torch.from_numpy(g["scheme/B"]).cuda())
    assert_bits(Y, g["scheme/Y"], "Scheme.matmul")


def _close(got, want, what, rel=1e-6, exact_frac=0.99):
    """All elements within `rel` of the output's scale except the few a one-ulp probability difference moved across
    a quantization boundary; at least `exact_frac` of them bit-identical."""
    got, want = np.asarray(got, np.float32), np.asarray(want, np.float32)
    same = got.view(np.uint32) == want.view(np.uint32)
    frac = same.mean()
    scale = np.abs(want).max()
    err = np.abs(got.astype(np.float64) - want.astype(np.float64)) / scale
    assert frac >= exact_frac, f"{what}: only {frac:.4f} of the elements are bit-identical"
    return float(err.max()), float(frac)


def test_attend_golden():
    from mxq.nn import attend
    g = golden("nn")
    q, k, v, mask = (torch.from_numpy(g[f"attend/{n}"]).cuda() for n in ("q", "k", "v", "mask"))
    s = hw_scheme()
    for key, kw in (("attend/o", dict(mask=mask)), ("attend/o_nomask", dict(mask=None)),
                    ("attend/o_chunk4", dict(mask=mask, chunk=4))):
        o = attend(q, k, v, kw["mask"], 32 ** -0.5, s, s, chunk=kw.get("chunk"))
        err, frac = _close(o.cpu().numpy(), g[key], key, exact_frac=0.999)
        assert err <= 1e-6, f"{key}: {err} (bit-identical fraction {frac})"


@pytest.mark.parametrize("B,H,Hkv,Tq,Tk,D,masked", [(2, 4, 4, 40, 40, 32, True), (3, 8, 2, 33, 50, 64, False),
                                                     (2, 6, 3, 17, 17, 32, "per-row")])
def test_attend_stacked_equals_loop(B, H, Hkv, Tq, Tk, D, masked):
    """The stacked path (Schemes of this package's quantizers and systolic: every head in one launch) against the
    per-head loop (the same Schemes with the quantizers wrapped, so they are not recognised) bit for bit: with and
    without a mask, a per-batch-row mask, grouped KV heads, Tq != Tk."""
    import mxq
    from mxq import Scheme, block, matmul, schedule
    from mxq.nn import attend
    g = torch.Generator().manual_seed(B * 100 + H)
    q = torch.randn(B, H, Tq, D, generator=g).cuda()
    k = torch.randn(B, Hkv, Tk, D, generator=g).cuda()
    v = torch.randn(B, Hkv, Tk, D, generator=g).cuda()
    mask = None
    if masked:
        rows = B if masked == "per-row" else 1
        m = torch.zeros(rows, 1, Tq, Tk)
        m[..., Tk // 2:] = float("-inf")
        m[..., 3] = -1.5
        mask = m.cuda()
    fast = hw_scheme()
    q8 = partial(block.mxgemmini.quantize, fmt="MXFP8_E4M3", axis=0)
    slow = Scheme("wrapped", a=lambda V: q8(V), b=lambda V: q8(V), reduce=fast.reduce)
    from mxq.nn import _attention
    assert _attention._stacked(fast) is not None and _attention._stacked(slow) is None
    o1 = attend(q, k, v, mask, D ** -0.5, fast, fast)
    o2 = attend(q, k, v, mask, D ** -0.5, slow, slow)
    assert_bits(o1.cpu().numpy(), o2.cpu().numpy(), "stacked vs loop")


def test_patched_llama():
    from transformers import LlamaConfig, LlamaForCausalLM
    from mxq.nn import patch
    g = golden("model")
    cfg = LlamaConfig(hidden_size=128, intermediate_size=352, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=4, head_dim=32, vocab_size=256, max_position_embeddings=128,
                      initializer_range=0.02)
    torch.manual_seed(0)
    model = LlamaForCausalLM(cfg).float().eval()
    ids = torch.from_numpy(g["ids"])
    model = model.cuda()
    with torch.no_grad():
        plain = model(ids.cuda()).logits.cpu().numpy()
    assert np.abs(plain - g["logits_plain"]).max() <= 1e-4 * np.abs(g["logits_plain"]).max()   # same weights
    s = hw_scheme()
    handle = patch(model, [("lm_head", None), ("model.layers.*.self_attn", (s, s)), (torch.nn.Linear, s)])
    mods = {n: m for n, m in model.named_modules() if type(m).__name__ == "MXLinear"}
    assert len(mods) == 2 * 7
    for name, mod in mods.items():                  # every MXLinear on the reference's own input
        x = torch.from_numpy(g[name + "/x"]).cuda()
        assert_bits(mod(x), g[name + "/y"], name)
    with torch.no_grad():
        logits = model(ids.cuda()).logits.cpu().numpy()
    rel = np.abs(logits.astype(np.float64) - g["logits"]).max() / np.abs(g["logits"]).max()
    assert rel <= 1e-6, rel                         # the north star's tolerance for the float32 glue
    handle.revert()
    assert not any(type(m).__name__ == "MXLinear" for m in model.modules())
