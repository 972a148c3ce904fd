"""The rest of the public API on the GPU against the reference's own outputs (tests/golden/api.npz):
the rounding modules' bits / integer forms (int64 results with carries past bit 31 kept), block.compose with the
reference's scale_factor / element_quant callables and the blocking helpers (bit for bit), the vector ops and
attend on decode, grouped-query and multi-chunk causal shapes, patch's dry-run tables (text), vector settings
through patch on a small Llama, and the Schemes MXQConfig builds (bit for bit through MXLinear).

Tolerances: float32 glue (torch's softmax / RMSNorm on the GPU sums in another order than on the CPU) as in
test_gpu_nn: outputs within 1e-6 of their scale, at least 99.9% bit-identical. With vector="bf16" every glue step
is rounded to bf16, so a one-ulp float32 difference from the GPU's exp or rsqrt that straddles a bf16 rounding
boundary moves that value by one bf16 step (2^-8 relative): vector results are held to 99% bit-identical and one
bf16 step (4e-3 of the scale), and whole-model logits under vector settings to 2e-2 of their scale."""
import json
from functools import partial

import numpy as np
import pytest
import torch

from _util import assert_bits, golden

pytestmark = pytest.mark.gpu


def _g():
    return golden("api")


def _msgs():
    return json.loads(str(_g()["msgs"]))


def _cuda(a, dtype=None):
    t = torch.from_numpy(np.asarray(a)).cuda()
    return t if dtype is None else t.to(dtype)


def hw_scheme(name="hw"):
    from mxq import Scheme, block, matmul, schedule
    q8 = partial(block.mxgemmini.quantize, fmt="MXFP8_E4M3", axis=0)
    return Scheme(name, a=q8, b=q8, reduce=partial(matmul.systolic, arith=matmul.MXGEMMINI(), schedule=schedule.HW_FINAL))


def _close(got, want, what, rel, exact_frac):
    """NaN where the reference has NaN (a query row whose keys are all masked under vector="bf16": the mask rounds to
    -inf and -inf - -inf is NaN, in the reference too); elsewhere within `rel` of the scale and at least
    `exact_frac` of the elements bit-identical."""
    got, want = np.asarray(got, np.float32), np.asarray(want, np.float32)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan), f"{what}: NaN positions differ"
    got, want = got[~nan], want[~nan]
    frac = float((got.view(np.uint32) == want.view(np.uint32)).mean()) if got.size else 1.0
    err = float((np.abs(got.astype(np.float64) - want) / max(np.abs(want).max(), 1e-30)).max()) if got.size else 0.0
    assert frac >= exact_frac and err <= rel, f"{what}: bit-identical {frac:.5f}, max error {err:.3g} of the scale"


def test_rounding_modules():
    from mxq import rounding
    g = _g()
    bt = _cuda(g["rbits/bits"])
    keep = torch.from_numpy(g["rbits/keep"]).cuda()
    for name in ("rne", "ties_away", "truncate"):
        mod = getattr(rounding, name)
        for k in (0, 3, 7, 10, 22):
            drop = 23 - k
            assert_bits(mod.bits(bt, drop, (1 << drop) - 1, 1 << (drop - 1)), g[f"rbits/{name}/{k}"], f"{name} keep {k}")
        drop = 23 - keep
        one = torch.ones((), dtype=torch.int64, device="cuda")
        mask, half = torch.bitwise_left_shift(one, drop) - 1, torch.bitwise_left_shift(one, drop - 1)
        assert_bits(mod.bits(bt, drop, mask, half), g[f"rbits/{name}/tensor"], f"{name} per-element keep")
        kk = g["rint/in"]
        assert_bits(mod.integer(_cuda(kk)), g[f"rint/{name}/f32"], f"{name} integer f32")
        assert_bits(mod.integer(_cuda(kk, torch.float64) * 1.5), g[f"rint/{name}/f64"], f"{name} integer f64")


def _steps():
    from mxq import scale_factor
    from mxq.element_quant import float_em, microsoft
    return {
        "mxquant_hwfloor": (partial(scale_factor.mxquant, floor=2.0 ** -23),
                            partial(float_em.quantize, e=4, m=3, rounding_mode="ties_away", grid="qtorch")),
        "ocp_microsoft": (partial(scale_factor.ocp, emax=8), partial(microsoft.quantize, fmt="MXFP8_E4M3")),
        "mxquant_ocp_rne": (scale_factor.mxquant, partial(float_em.quantize, e=3, m=2, rounding_mode="rne",
                                                           grid="ocp")),
        "below_top": (partial(scale_factor.ocp_below_top, emax=4),
                      partial(microsoft.quantize, fmt="MXFP6_E3M2", rounding_mode="nearest")),
        "no_clip": (partial(scale_factor.ocp_no_clip, fmt="MXFP6_E2M3"), partial(microsoft.quantize, fmt="MXFP6_E2M3")),
        "ieee_truncate": (partial(scale_factor.ocp, emax=15, scale_bits=5),
                          partial(float_em.quantize, e=5, m=2, rounding_mode="truncate", grid="ieee")),
        "no_scale": (None, partial(float_em.quantize, e=4, m=3, rounding_mode="rne", grid="ocp")),
        "no_elem": (scale_factor.mxquant, None),
        "neither": (None, None),
    }


def test_compose_with_reference_steps():
    from mxq import block
    g = _g()
    V = _cuda(g["compose/V"])
    for name, (sc, el) in _steps().items():
        for axis, bs in ((0, 32), (1, 32), (1, 16), (2, 4), (-1, 3), (1, 7)):
            P, X = block.compose(V, scale=sc, elem=el, axis=axis, block_size=bs)
            assert_bits(P, g[f"compose/{name}/{axis}/{bs}/P"], f"compose {name} axis {axis} block {bs} P")
            assert_bits(X, g[f"compose/{name}/{axis}/{bs}/X"], f"compose {name} axis {axis} block {bs} X")


def test_blocking_helpers():
    from mxq import block
    from mxq.block import _driver
    g = _g()
    V = _cuda(g["compose/V"])
    for axis, bs in ((0, 32), (1, 16), (1, 7), (2, 4)):
        b = _driver.to_blocks(V, axis, bs)
        assert_bits(b.data, g[f"blocks/{axis}/{bs}/data"], f"to_blocks axis {axis} block {bs}")
        assert_bits(_driver.codes_from_blocks(b.data * 2 + 1, b), g[f"blocks/{axis}/{bs}/codes"], "codes_from_blocks")
        X = _driver.scales_from_blocks(b.data.abs().amax(-1, keepdim=True), b)
        assert_bits(X, g[f"blocks/{axis}/{bs}/scales"], "scales_from_blocks")
        assert_bits(block.dequantize(V, X, axis=axis, block_size=bs), g[f"blocks/{axis}/{bs}/dequantize"], "dequantize")


def test_vector_ops():
    from mxq.nn import _vector
    g = _g()
    _close(_vector.softmax(_cuda(g["vector/S"]), "bf16").cpu(), g["vector/softmax_bf16"], "softmax bf16", 4e-3, 0.99)
    x, w = _cuda(g["vector/x"]), _cuda(g["vector/w"])
    _close(_vector.rmsnorm(x, w, 1e-6, "bf16").cpu(), g["vector/rmsnorm_bf16"], "rmsnorm bf16", 4e-3, 0.99)
    _close(_vector.rmsnorm(x, w, 1e-6, None).cpu(), g["vector/rmsnorm_none"], "rmsnorm", 1e-6, 0.0)   # GPU rsqrt


@pytest.mark.parametrize("shape,chunk", [("decode", None), ("gqa4", None), ("causal_chunks", 16),
                                         ("padded_chunks", 8)])
def test_attend_shapes(shape, chunk):
    """Decode (one query over 23 keys), four query heads per KV head, and multi-chunk causal / left-padded masks
    (where the reference skips the key blocks a chunk's mask removes), each on both paths of attend: the stacked
    one (every head in one launch) and the per-head loop (Schemes it does not recognise)."""
    from mxq import Scheme
    from mxq.nn import attend
    g = _g()
    q, k, v, mask = (_cuda(g[f"attend/{shape}/{n}"]) for n in ("q", "k", "v", "mask"))
    fast = hw_scheme()
    slow = Scheme("wrapped", a=lambda V: fast.a(V), b=lambda V: fast.b(V), reduce=fast.reduce)
    for s in (fast, slow):
        o = attend(q, k, v, mask, 32 ** -0.5, s, s, chunk=chunk)
        _close(o.cpu(), g[f"attend/{shape}/o"], f"attend {shape} ({s.name})", 1e-6, 0.999)
        o = attend(q, k, v, mask, 32 ** -0.5, s, s, chunk=chunk, vector="bf16")
        _close(o.cpu(), g[f"attend/{shape}/o_bf16"], f"attend {shape} bf16 ({s.name})", 4e-3, 0.99)


def _tiny_llama():
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(hidden_size=64, intermediate_size=96, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=16, vocab_size=128, max_position_embeddings=64,
                      initializer_range=0.02)
    torch.manual_seed(0)
    return LlamaForCausalLM(cfg).float().eval()


def test_patch_vector_settings(capsys):
    from mxq.nn import is_attention, patch
    g, m = _g(), _msgs()
    hw = hw_scheme()
    settings = {"bf16": ([("lm_head", None), ("model.layers.*.self_attn", (hw, hw)), (torch.nn.Linear, hw)], "bf16"),
                "rmsnorm": ([("lm_head", None), (torch.nn.Linear, hw)], {"rmsnorm": "bf16"}),
                "softmax_exact": ([("lm_head", None), (is_attention, None), (torch.nn.Linear, hw)],
                                  {"softmax": "bf16"})}
    ids = _cuda(g["model/ids"])
    for name, (rules, vec) in settings.items():
        model = _tiny_llama().cuda()
        capsys.readouterr()
        patch(model, rules, dry_run=True, vector=vec)
        assert capsys.readouterr().out == m[f"patch/{name}/dry_run"], name
        assert not any(type(x).__name__ == "MXLinear" for x in model.modules())      # dry run: nothing changed
        handle = patch(model, rules, vector=vec)
        with torch.no_grad():
            logits = model(ids).logits.cpu()
        _close(logits, g[f"model/{name}/logits"], f"logits {name}", 2e-2, 0.0)
        handle.revert()
        assert not any(type(x).__name__ == "MXLinear" for x in model.modules())
        assert all("forward" not in x.__dict__ for x in model.modules() if type(x).__name__.endswith("RMSNorm"))
        with torch.no_grad():
            plain = model(ids).logits.cpu()
        _close(plain, g[f"model/{name}/logits_reverted"], f"reverted {name}", 1e-4, 0.0)


def test_patch_shared_modules_tables(capsys):
    from test_api_host import _Shared, _Twice
    from mxq.nn import is_attention, patch
    m = _msgs()
    hw = hw_scheme()
    capsys.readouterr()
    patch(_Twice().cuda(), [("c", None), (torch.nn.Linear, hw)], dry_run=True)
    assert capsys.readouterr().out == m["patch/twice/dry_run"]
    patch(_Shared().cuda(), [("*.c", None), ("*.att", (hw, hw)), (is_attention, None), (torch.nn.Linear, hw)],
          dry_run=True, vector={"rmsnorm": None, "softmax": "bf16"})
    assert capsys.readouterr().out == m["patch/shared/dry_run"]
    model = _Shared().cuda()
    lin = model.x.a
    handle = patch(model, [("*.c", None), (torch.nn.Linear, hw)])
    # a and b are two attributes holding one Linear: each gets an MXLinear, both on the layer's own Parameter;
    # x and y are one subtree, so x.a and y.a are one attribute and one MXLinear
    assert type(model.x.a).__name__ == "MXLinear" and type(model.x.b).__name__ == "MXLinear"
    assert model.x.a.weight is lin.weight and model.x.b.weight is lin.weight and model.y.a is model.x.a
    assert type(model.x.c).__name__ == "Linear"
    handle.revert()
    assert model.x.a is lin and model.x.b is lin


@pytest.mark.parametrize("name", ["default", "e2m3_truncate", "prod44_nofloor", "exact", "lut", "size8", "via"])
def test_mxqconfig_schemes(name):
    from test_api_host import CONFIGS
    from mxq.nn import MXLinear
    from mxq.nn.torchao import MXQConfig, apply
    g = _g()
    lin = torch.nn.Linear(64, 24)
    with torch.no_grad():
        lin.weight.copy_(torch.from_numpy(g["torchao/W"]))
        lin.bias.copy_(torch.from_numpy(g["torchao/b"]))
    lin = lin.cuda()
    x = _cuda(g["torchao/x"])
    c = MXQConfig(**CONFIGS[name])
    assert_bits(MXLinear(lin, c.scheme(lin.weight.device), chunk=c.chunk)(x), g[f"torchao/{name}/y"], name)
    assert apply(lin, c) is lin                                   # in place, as the torchao handler
    with torch.no_grad():
        assert_bits(lin(x), g[f"torchao/{name}/y"], f"{name} through apply")


@pytest.mark.parametrize("vector", [None, "bf16"])
def test_attend_masked_skip_is_bit_identical(monkeypatch, vector):
    """Multi-chunk causal and left-padded masks: chunks whose mask removes key blocks skip them (checked by
    watching the live ranges), and the output is bit for bit that of one chunk (where nothing is skipped), on the
    stacked path and the per-head loop. A -1e4 mask (older HF) is never skipped."""
    from mxq import Scheme
    from mxq.nn import _attention, attend
    ranges = []
    real = _attention._live_keys
    monkeypatch.setattr(_attention, "_live_keys", lambda *a: ranges.append(real(*a)) or ranges[-1])
    g = torch.Generator().manual_seed(31)
    B, H, Hkv, T, D = 2, 4, 2, 96, 32
    q, k, v = (torch.randn(B, h, T, D, generator=g).cuda() for h in (H, Hkv, Hkv))
    fmin = torch.finfo(torch.float32).min
    causal = torch.triu(torch.full((T, T), fmin), diagonal=1)[None, None].repeat(B, 1, 1, 1).cuda()
    causal[1, :, :, :40] = fmin                                    # batch row 1 left-padded by 40 keys
    causal[1, :, :40, :] = fmin                                    # (its padded queries see nothing: uniform rows)
    fast = hw_scheme()
    slow = Scheme("wrapped", a=lambda V: fast.a(V), b=lambda V: fast.b(V), reduce=fast.reduce)
    for s in (fast, slow):
        ranges.clear()
        chunked = attend(q, k, v, causal, D ** -0.5, s, s, chunk=16, vector=vector)
        assert any(hi - lo < T for lo, hi in ranges), (s.name, ranges)
        whole = attend(q, k, v, causal, D ** -0.5, s, s, chunk=T, vector=vector)
        assert_bits(chunked, whole, f"skipped vs whole ({s.name})")
        ranges.clear()
        soft = torch.where(causal == fmin, torch.tensor(-1e4, device="cuda"), causal)
        attend(q, k, v, soft, D ** -0.5, s, s, chunk=16, vector=vector)
        assert all((lo, hi) == (0, T) for lo, hi in ranges), (s.name, ranges)
