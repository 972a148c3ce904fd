"""mxq.nn.torchao — MXLinear behind TorchAO's `quantize_` (mxq/nn/torchao.py:43-145 of the reference): one Scheme
as plain fields, so a checkpoint's config.json can carry it.

    cfg = MXQConfig(fmt="MXFP8_E4M3", prod=[4, 3], prod_floor=-16, ladder=[[4, 4]] * 8 + ..., size=16)
    quantize_(model, cfg)                 # with torchao installed: the handler below is registered for MXQConfig
    apply(linear, cfg)                    # the same handler, callable without torchao

Fields -> Scheme:
    fmt, rounding_mode, scale_floor, via, block_size   block.mxgemmini.quantize of both operands (axis 0)
    lut {"group": G, "max_iters": n}                   block.lut.quantize instead (rows = 2^G)
    prod, prod_floor, ladder, size                     matmul.systolic(MXGEMMINI(*prod, prod_floor), ladder, size)
    reduce "exact"                                     fp64_accum instead of the systolic column
    compiled                                           None: compiled on a CUDA layer; matmul.compiled is the same
                                                       Arithmetic here (the kernels are the fusion), so it changes
                                                       nothing but is kept and validated as a field
    chunk, name                                        MXLinear's token chunk, the Scheme's name

Lists throughout (torchao's encoder refuses tuples; tuples given are turned into lists). torchao itself is not a
dependency of this package: without it MXQConfig is a plain dataclass and `apply` does what the registered handler
would.
"""
from dataclasses import asdict, dataclass, field
from functools import partial
from typing import Dict, List, Optional

import torch
from torch import nn

from .. import block, lut, matmul, scale_factor
from .._fp64_accum import fp64_accum
from ..element_quant.formats import get
from ..schedule import HW_FINAL
from ..scheme import Scheme
from ._linear import MXLinear

try:                                                     # optional: the base class and handler registry
    from torchao.core.config import AOBaseConfig as _Base
    from torchao.quantization.transform_module import register_quantize_module_handler as _register
except ImportError:                                      # torchao is absent: a plain base, no registry
    _Base = object
    _register = None

__all__ = ["MXQConfig", "apply"]

REDUCERS = ("hardware", "exact")


def _whole(v) -> bool:
    return isinstance(v, int) and not isinstance(v, bool)


def _em(v, what: str) -> List[int]:
    """[e, m]: two positive integers (a list or tuple given, a list kept)."""
    v = list(v) if isinstance(v, (list, tuple)) else v
    if isinstance(v, list) and len(v) == 2 and all(_whole(x) and x > 0 for x in v):
        return v
    raise ValueError(f"MXQConfig: {what} {v!r} must be two positive integers [e, m]")


@dataclass
class MXQConfig(_Base):
    """One Scheme as fields; the defaults are the MX-Gemmini tapeout (RNE, the 2^-23 block-max floor, E4M3
    products flushed below 2^-16, the HW_FINAL ladder, a 16-deep column)."""
    fmt: str = "MXFP8_E4M3"
    rounding_mode: str = "rne"
    scale_floor: float = scale_factor.HARDWARE_FLOOR
    via: Optional[List[int]] = None
    block_size: int = 32
    prod: List[int] = field(default_factory=lambda: [4, 3])
    prod_floor: Optional[int] = -16
    ladder: List[List[int]] = field(default_factory=lambda: [[e, m] for e, m in HW_FINAL])
    size: int = 16
    reduce: str = "hardware"
    compiled: Optional[bool] = None
    chunk: Optional[int] = None
    name: str = "mxq"
    lut: Optional[Dict[str, int]] = None

    def __post_init__(self):
        fmt = get(self.fmt)                               # an unknown name raises the formats table's ValueError
        if fmt is None:
            raise ValueError("MXQConfig: fmt FP32 is no quantization; leave the layer out instead")
        if self.reduce not in REDUCERS:
            raise ValueError(f"MXQConfig: reduce {self.reduce!r}; choose from {', '.join(REDUCERS)}")
        self.prod = _em(self.prod, "prod")
        self.ladder = [_em(lane, f"ladder[{i}]") for i, lane in enumerate(self.ladder)]
        if self.via is not None:
            self.via = _em(self.via, "via")
        if len(self.ladder) != self.size:
            raise ValueError(f"MXQConfig: ladder has {len(self.ladder)} lanes for a {self.size}-deep column "
                             "(one accumulator format per lane)")
        if not (self.prod_floor is None or _whole(self.prod_floor)):
            raise ValueError(f"MXQConfig: prod_floor {self.prod_floor!r} must be an integer exponent or None")
        if not _whole(self.block_size) or self.block_size < 1 or self.block_size % self.size:
            raise ValueError(f"MXQConfig: block_size {self.block_size!r} must be a multiple of size {self.size}")
        if not (self.compiled is None or isinstance(self.compiled, bool)):
            raise ValueError(f"MXQConfig: compiled {self.compiled!r} must be True, False or None")
        if not (self.chunk is None or (_whole(self.chunk) and self.chunk >= 1)):
            raise ValueError(f"MXQConfig: chunk {self.chunk!r} must be a positive integer or None")
        if self.lut is not None:
            ok = (isinstance(self.lut, dict) and set(self.lut) == {"group", "max_iters"}
                  and all(_whole(v) and v >= 0 for v in self.lut.values()))
            if not ok:
                raise ValueError(f"MXQConfig: lut {self.lut!r} must be {{'group': G, 'max_iters': n}}, "
                                 "non-negative integers")
            if fmt.name not in lut.FORMATS:
                raise ValueError(f"MXQConfig: fmt {self.fmt} has no LUT on MX-Gemmini; LUT formats: "
                                 f"{', '.join(lut.FORMATS)}")
            if self.via is not None:
                raise ValueError("MXQConfig: via is the fp4 requantizer's rounding; a LUT operand has none")
            self.lut = dict(self.lut)

    def scheme(self, device=None) -> Scheme:
        """The Scheme of these fields for a layer on `device`. One Scheme per config and compile setting is kept and
        reused while the fields are unchanged (every layer a config converts shares it)."""
        compile = self.compiled if self.compiled is not None else torch.device(device or "cpu").type == "cuda"
        fields = asdict(self)
        memo = self.__dict__.setdefault("_schemes", {})   # not a field: asdict and to_dict do not see it
        hit = memo.get(compile)
        if hit is not None and hit[0] == fields:
            return hit[1]
        common = dict(fmt=self.fmt, axis=0, block_size=self.block_size, rounding_mode=self.rounding_mode,
                      scale_floor=self.scale_floor)
        if self.lut is None:
            quantize = partial(block.mxgemmini.quantize, **common,
                               via=None if self.via is None else tuple(self.via))
            rows = 1
        else:
            quantize = partial(block.lut.quantize, **common, group=self.lut["group"],
                               max_iters=self.lut["max_iters"])
            rows = 1 << self.lut["group"]
        if self.reduce == "exact":
            reduce = partial(fp64_accum, block_size=self.block_size)
        else:
            arith = matmul.MXGEMMINI(*self.prod, prod_floor=self.prod_floor)
            if compile:
                arith = matmul.compiled(arith)
            reduce = partial(matmul.systolic, arith=arith, schedule=[tuple(lane) for lane in self.ladder],
                             size=self.size, block_size=self.block_size)
        made = Scheme(self.name, a=quantize, b=quantize, reduce=reduce, rows=rows, block_size=self.block_size)
        memo[compile] = (fields, made)
        return made

    @classmethod
    def from_dict(cls, d: dict) -> "MXQConfig":
        """Rebuild from torchao's `config_to_dict(cfg)` (or its "_data" part, or to_dict())."""
        if isinstance(d, dict) and d.get("_type", cls.__name__) != cls.__name__:
            raise ValueError(f"MXQConfig.from_dict: this dict is a {d['_type']}")
        data = d.get("_data", d) if isinstance(d, dict) else d
        return cls(**data)

    def to_dict(self) -> dict:
        return asdict(self)


def apply(module: nn.Module, config: MXQConfig) -> nn.Module:
    """Route this Linear's forward through an MXLinear sharing its weight and bias, in place; returns the same
    object (Hugging Face drops a handler's replacement module without an error, so the module itself changes)."""
    if not isinstance(module, nn.Linear):
        raise TypeError(f"MXQConfig applies to nn.Linear, got {type(module).__name__}")
    runner = MXLinear(module, config.scheme(module.weight.device), chunk=config.chunk)
    object.__setattr__(module, "_mxq", runner)            # not a registered child: no duplicate parameters
    module.forward = runner.forward
    return module


if _register is not None:
    _register(MXQConfig)(apply)
