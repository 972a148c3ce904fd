"""The host-side parts of the public API against the reference's own outputs (tests/golden/api.npz), on the CPU:
schedule.load / fixed (results and every error message), patch's refusals (all raised before any Scheme runs or
any layer is touched), and mxq.nn.torchao.MXQConfig (fields, validation messages, to_dict / from_dict, the Scheme
it builds)."""
import json
import os

import pytest
import torch

from _util import golden


def _msgs():
    return json.loads(str(golden("api")["msgs"]))


def test_schedule_load_and_fixed(tmp_path):
    from mxq import schedule
    m = _msgs()
    for name, text in m["schedule/csv"].items():
        path = os.path.join(tmp_path, name + ".csv")
        with open(path, "w") as f:
            f.write(text)
        want = m[f"schedule/{name}"]
        if "ok" in want:
            assert [list(x) for x in schedule.load(path, rows=want["rows"])] == want["ok"], name
        else:
            with pytest.raises(ValueError) as e:
                schedule.load(path, rows=want["rows"])
            assert str(e.value).replace(path, "<path>") == want["error"], name
    assert [list(x) for x in schedule.fixed(5, 6, rows=4)] == m["schedule/fixed"]
    assert schedule.HW_FINAL == [(4, 4)] * 8 + [(4, 5)] * 2 + [(4, 6)] * 5 + [(8, 7)]


class _Twice(torch.nn.Module):
    """One Linear held in two attributes, another once, and an attention module (q_proj and k_proj)."""

    def __init__(self):
        super().__init__()
        self.a = torch.nn.Linear(32, 16)
        self.b = self.a
        self.c = torch.nn.Linear(16, 8)
        self.att = torch.nn.Module()
        self.att.q_proj = torch.nn.Linear(32, 32)
        self.att.k_proj = torch.nn.Linear(32, 32)


class _Shared(torch.nn.Module):
    """A whole subtree held twice: each of its Linear attributes is reachable under two names."""

    def __init__(self):
        super().__init__()
        self.x = _Twice()
        self.y = self.x


def test_patch_refusals():
    from functools import partial
    from mxq import Scheme, block, matmul, schedule
    from mxq.nn import patch
    q8 = partial(block.mxgemmini.quantize, fmt="MXFP8_E4M3", axis=0)
    hw = Scheme("hw", a=q8, b=q8, reduce=partial(matmul.systolic, arith=matmul.MXGEMMINI(), schedule=schedule.HW_FINAL))
    cases = {
        "bad_rule": lambda: patch(_Twice(), [("a", "fp8")]),
        "no_linear": lambda: patch(_Twice(), [("nothing.*", hw), (torch.nn.Linear, None)]),
        "hidden": lambda: patch(_Twice(), [(torch.nn.Linear, None), ("c", hw)]),
        "no_core": lambda: patch(_Twice(), [("x", (hw, hw))]),
        "softmax_no_attention": lambda: patch(_Twice(), [], vector="bf16"),
        "vector_spelling": lambda: patch(_Twice(), [], vector={"softmax": "fp16"}),
        "same_site": lambda: patch(_Shared(), [("x.c", hw), ("y.c", None), (torch.nn.Linear, None)]),
        "same_core": lambda: patch(_Shared(), [("x.att", (hw, hw)), (torch.nn.Linear, None)]),
    }
    m = _msgs()
    for name, fn in cases.items():
        with pytest.raises(ValueError) as e:
            fn()
        assert str(e.value) == m[f"patch_error/{name}"], name


def test_patch_refusal_leaves_model_alone():
    from mxq.nn import patch
    model = _Shared()
    before = [(n, id(mod)) for n, mod in model.named_modules(remove_duplicate=False)]
    with pytest.raises(ValueError):
        patch(model, [("x.c", None), ("nothing", None)])
    assert [(n, id(mod)) for n, mod in model.named_modules(remove_duplicate=False)] == before


CONFIGS = {
    "default": {},
    "e2m3_truncate": {"fmt": "MXFP6_E2M3", "rounding_mode": "truncate", "scale_floor": 1e-38},
    "prod44_nofloor": {"prod": (4, 4), "prod_floor": None, "ladder": [[8, 7]] * 16},
    "exact": {"reduce": "exact"},
    "lut": {"fmt": "MXFP6_E3M2", "lut": {"group": 1, "max_iters": 5}},
    "size8": {"size": 8, "ladder": [[4, 6]] * 8, "block_size": 32, "chunk": 3},
    "via": {"fmt": "MXFP4", "via": [3, 1]},
}
BAD = {
    "fp32": {"fmt": "FP32"}, "reduce": {"reduce": "fast"}, "prod": {"prod": [4]},
    "ladder_len": {"ladder": [[4, 4]] * 15}, "prod_floor": {"prod_floor": 1.5},
    "block": {"block_size": 24}, "compiled": {"compiled": 1}, "chunk": {"chunk": 0},
    "lut_keys": {"fmt": "MXFP6_E3M2", "lut": {"group": 1}},
    "lut_fmt": {"fmt": "MXFP4", "lut": {"group": 1, "max_iters": 2}},
    "lut_via": {"fmt": "MXFP6_E3M2", "via": [3, 1], "lut": {"group": 1, "max_iters": 2}},
    "ladder_entry": {"ladder": [[4, 4]] * 15 + [[4, 0]]},
}


def test_mxqconfig_fields_and_scheme():
    from mxq.nn.torchao import MXQConfig
    m = _msgs()
    for name, kw in CONFIGS.items():
        c = MXQConfig(**kw)
        assert c.to_dict() == m[f"torchao/{name}/dict"], name
        s = c.scheme("cpu")
        assert {"name": s.name, "rows": s.rows, "block_size": s.block_size} == m[f"torchao/{name}/scheme"], name
        assert c.scheme("cpu") is s                                     # one Scheme per config and setting
        c.size = c.size                                                 # unchanged fields: still the same
        assert c.scheme("cpu") is s
    for name, kw in BAD.items():
        with pytest.raises(ValueError) as e:
            MXQConfig(**kw)
        assert str(e.value) == m[f"torchao_error/{name}"], name
    with pytest.raises(ValueError) as e:
        MXQConfig.from_dict({"_type": "Other", "_data": {}})
    assert str(e.value) == m["torchao_error/from_dict_type"]
    rt = MXQConfig.from_dict({"_type": "MXQConfig", "_data": MXQConfig(fmt="MXFP8_E5M2").to_dict()})
    assert rt.to_dict() == m["torchao/roundtrip"]


def test_mxqconfig_apply_refuses_non_linear():
    from mxq.nn.torchao import MXQConfig, apply
    with pytest.raises(TypeError, match="applies to nn.Linear"):
        apply(torch.nn.Conv1d(2, 2, 1), MXQConfig())


def test_stream_runs_cover_and_ramp():
    """The host-streaming chunk runs: contiguous, covering every unit once, none longer than the chunk, and short at
    both ends when there are enough units for the ramps."""
    from mxq.block._driver import _runs
    for total in (1, 2, 7, 10, 31, 53, 60, 100, 256, 1000):
        for per in (1, 2, 3, 8, 16, 64):
            r = _runs(total, per)
            assert r[0][0] == 0 and r[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(r, r[1:]))
            assert all(0 < b - a <= per for a, b in r)
            if total > 2 * (max(1, per >> 3) + max(1, per >> 2) + max(1, per >> 1)) + per:
                assert r[0][1] - r[0][0] == max(1, per >> 3) and r[-1][1] - r[-1][0] == max(1, per >> 3)
