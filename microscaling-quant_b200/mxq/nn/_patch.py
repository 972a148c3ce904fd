"""patch(model, rules): which Scheme each nn.Linear (and each attention core) runs through
(mxq/nn/_patch.py:123-287).

    rules = [("lm_head", None),                 # a layer name, * wildcards; None leaves the layer as it is
             ("*.mlp.down_proj", FP6),          # a Scheme
             (is_attention, None),              # a function (name, module, parent) -> bool
             (nn.Linear, FP8),                  # a layer type
             ("model.layers.*.self_attn", (QK, PV))]   # a pair of Schemes: that attention module's core
    handle = patch(model, rules)                # first matching rule wins
    handle.revert()
    patch(model, rules, dry_run=True)           # print the table, change nothing

Before anything is replaced every Scheme runs once on a tiny matmul (and every core on a tiny attention), so a bad
schedule or format fails here. A rule that chooses nothing raises. A layer reachable under several names is
replaced at every attribute holding it; two names of one attribute asking for different rules raise.
vector="bf16" (or {"softmax": ..., "rmsnorm": ...}) rounds the vector ops' steps to bf16: softmax runs in attend
(attention modules without a core rule get the EXACT core), and every *RMSNorm forward is replaced after a check
that the unrounded replacement reproduces the module's own output bit for bit.
"""
from fnmatch import fnmatchcase
from functools import partial
from typing import Callable, List, Optional, Sequence, Tuple, Union

import torch
from torch import nn

from ..scheme import Scheme
from ._attention import NAME as _CORE, attend, register
from ._linear import MXLinear
from ._vector import EXACT, resolve, rmsnorm

__all__ = ["patch", "is_attention", "Handle"]

Selector = Union[str, type, Callable[[str, nn.Module, nn.Module], bool]]
Rule = Tuple[Selector, Union[None, Scheme, Tuple[Scheme, Scheme]]]


def _is_core(value) -> bool:
    return isinstance(value, tuple) and len(value) == 2 and all(isinstance(s, Scheme) for s in value)


def _holds_core(module: nn.Module) -> bool:
    return hasattr(module, "q_proj") and hasattr(module, "k_proj")


def is_attention(name: str, module: nn.Module, parent: nn.Module) -> bool:
    """Is this Linear one of an attention module's projections? (its parent holds q_proj and k_proj)"""
    return hasattr(parent, "q_proj") and hasattr(parent, "k_proj")


def _smoke(scheme: Scheme) -> None:
    g = torch.Generator().manual_seed(0)
    n, K = 2 * scheme.rows, 3 * scheme.block_size          # two whole LUT groups, three blocks
    scheme.matmul(torch.randn(K, n, generator=g), torch.randn(K, n, generator=g))


def _smoke_core(qk: Scheme, pv: Scheme) -> None:
    g = torch.Generator().manual_seed(0)
    t = 2 * max(qk.block_size, pv.block_size) * max(qk.rows, pv.rows)
    q, k, v = (torch.randn(1, h, t, 32, generator=g) for h in (2, 1, 1))
    attend(q, k, v, None, 32 ** -0.5, qk, pv)


def _is_rmsnorm(module: nn.Module) -> bool:
    return type(module).__name__.endswith("RMSNorm")


def _eps(module: nn.Module) -> float:
    for attr in ("variance_epsilon", "eps"):
        if isinstance(getattr(module, attr, None), float):
            return getattr(module, attr)
    raise ValueError(f"{type(module).__name__}: no float variance_epsilon or eps attribute")


def _check_rmsnorm(name: str, module: nn.Module) -> float:
    weight = getattr(module, "weight", None)
    if not isinstance(weight, torch.Tensor) or weight.ndim != 1:
        raise ValueError(f"{name} ({type(module).__name__}): no 1-D weight, not the RMSNorm mxq knows")
    eps = _eps(module)
    g = torch.Generator().manual_seed(0)
    x = (torch.randn(3, weight.shape[0], generator=g) * 3).to(device=weight.device, dtype=weight.dtype)
    with torch.no_grad():
        theirs, ours = module(x), rmsnorm(x, weight, eps, None)
    if theirs.dtype != ours.dtype or not torch.equal(theirs, ours):
        raise ValueError(f"{name} ({type(module).__name__}) does not compute weight · x / sqrt(mean(x²) + eps) the way "
                         "transformers' LlamaRMSNorm does; vector rmsnorm cannot replace it")
    return eps


def _rmsnorm_forward(module: nn.Module, eps: float, precision: str, x: torch.Tensor) -> torch.Tensor:
    return rmsnorm(x, module.weight, eps, precision)


def _set_attention(model: nn.Module, name: str) -> None:
    if hasattr(model, "set_attn_implementation"):
        model.set_attn_implementation(name)
    else:
        model.config._attn_implementation = name


def _matches(selector: Selector, name: str, module: nn.Module, parent: nn.Module) -> bool:
    if isinstance(selector, str):
        return fnmatchcase(name, selector)
    if isinstance(selector, type):
        return isinstance(module, selector)
    return bool(selector(name, module, parent))


class Handle:
    """What patch did: `table` rows (layer name, in, out, rule index or None, Scheme name or None); `cores` rows
    (attention module name, rule index or None, (qk name, pv name) or None)."""

    def __init__(self, model, table, replaced, cores=None, cored=None, previous=None, vector=None, norms=None,
                 normed=None):
        self._model, self.table, self._replaced = model, table, replaced
        self.cores, self._cored, self._previous = cores or [], cored or [], previous
        self.vector, self.norms, self._normed = vector or resolve(None), norms or [], normed or []

    def revert(self) -> None:
        for parent, leaf, original in self._replaced:
            setattr(parent, leaf, original)
        self._replaced = []
        for module in self._cored:
            del module._mxq_core
            if hasattr(module, "_mxq_vector"):
                del module._mxq_vector
        if self._cored:
            _set_attention(self._model, self._previous)
        self._cored = []
        for module in self._normed:
            del module.forward
        self._normed = []

    def __str__(self) -> str:
        width = max([len(r[0]) for r in self.table] + [len(r[0]) for r in self.cores] + [5])
        lines = [f"{'layer':{width}s}  {'in':>6s} {'out':>6s}  rule  scheme"]
        for name, k, n, rule, scheme in self.table:
            lines.append(f"{name:{width}s}  {k:6d} {n:6d}  {'-' if rule is None else rule:>4}  "
                         f"{'no rule' if rule is None else (scheme or 'left as is')}")
        if any(names is not None for _, _, names in self.cores):
            lines.append(f"{'attention core':{width}s}  {'':13s}  rule  Q·Kᵀ, P·V")
            for name, rule, names in self.cores:
                lines.append(f"{name:{width}s}  {'':13s}  {'-' if rule is None else rule:>4}  "
                             f"{'sdpa (no rule)' if names is None else ', '.join(names)}"
                             f"{'  (vector softmax)' if rule is None and names is not None else ''}")
        if any(self.vector.values()):
            n = {"softmax": sum(names is not None for _, _, names in self.cores), "rmsnorm": len(self.norms)}
            lines.append("vector  " + ", ".join(f"{op} {p or 'as transformers'}" + (f" ({n[op]} modules)" if p else "")
                                                for op, p in self.vector.items()))
        return "\n".join(lines)


def patch(model: nn.Module, rules: Sequence[Rule], chunk: Optional[int] = None, dry_run: bool = False,
          cache_weights: bool = True, vector=None) -> Handle:
    vector = resolve(vector)
    for i, rule in enumerate(rules):
        if len(rule) != 2 or not (rule[1] is None or isinstance(rule[1], Scheme) or _is_core(rule[1])):
            raise ValueError(f"rule {i} must be (selector, Scheme or None or (qk Scheme, pv Scheme)), got {rule!r}")
    linear_rules = [i for i, (_, v) in enumerate(rules) if not _is_core(v)]
    core_rules = [i for i, (_, v) in enumerate(rules) if _is_core(v)]

    walk = list(model.named_modules(remove_duplicate=False))           # a module held twice is seen under both
    holder = {name: module for name, module in walk}

    def parent_of(name):
        return holder[name.rpartition(".")[0]]

    chosen = [(name, mod, parent_of(name),
               next((i for i in linear_rules if _matches(rules[i][0], name, mod, parent_of(name))), None))
              for name, mod in walk if name and isinstance(mod, nn.Linear)]
    cores = [(name, mod, next((i for i in core_rules if _matches(rules[i][0], name, mod, parent_of(name))), None))
             for name, mod in walk if name and _holds_core(mod)]
    unused = [i for i in linear_rules if all(hit != i for *_, hit in chosen)]
    if unused:
        raise ValueError(f"rules {unused} choose no Linear layer (misspelt, or hidden behind an earlier rule): "
                         f"{[rules[i][0] for i in unused]}")
    unused = [i for i in core_rules if all(hit != i for *_, hit in cores)]
    if unused:
        raise ValueError(f"rules {unused} choose no attention module (one holding q_proj and k_proj): "
                         f"{[rules[i][0] for i in unused]}")
    for module in {id(m): m for _, m, hit in cores if hit is not None}.values():
        if len({hit for _, m, hit in cores if m is module}) > 1:
            raise ValueError(f"{[n for n, m, _ in cores if m is module]} are the same attention module but match "
                             "different rules; one of them has to go")

    sites: dict = {}                                                  # one attribute = one place a layer runs
    for row in chosen:
        name, _, parent, _ = row
        sites.setdefault((id(parent), name.rpartition(".")[2]), []).append(row)
    for rows_ in sites.values():
        if len({r[3] for r in rows_}) > 1:
            raise ValueError(f"{[r[0] for r in rows_]} are the same layer but match different rules "
                             f"{[r[3] for r in rows_]}; one of them has to go")

    if vector["softmax"] and not cores:
        raise ValueError("vector softmax: the model has no attention module (one holding q_proj and k_proj)")
    norms = list({id(m): (n, m) for n, m in walk if n and _is_rmsnorm(m)}.values()) if vector["rmsnorm"] else []
    if vector["rmsnorm"] and not norms:
        raise ValueError("vector rmsnorm: the model has no module whose class name ends in RMSNorm")

    for i in linear_rules:                                            # fail now, not mid-run
        if rules[i][1] is not None:
            _smoke(rules[i][1])
    for i in core_rules:
        _smoke_core(*rules[i][1])
    if vector["softmax"] and any(hit is None for *_, hit in cores):
        _smoke_core(EXACT, EXACT)
    eps = [_check_rmsnorm(n, m) for n, m in norms]

    table = [(name, m.in_features, m.out_features, hit,
              None if hit is None or rules[hit][1] is None else rules[hit][1].name) for name, m, _, hit in chosen]

    def core_of(hit):
        return rules[hit][1] if hit is not None else (EXACT, EXACT) if vector["softmax"] else None

    core_table = [(name, hit, None if core_of(hit) is None else tuple(s.name for s in core_of(hit)))
                  for name, _, hit in cores]
    replaced = []
    if not dry_run:
        for rows_ in sites.values():
            name, module, parent, hit = rows_[0]
            if hit is None or rules[hit][1] is None:
                continue
            leaf = name.rpartition(".")[2]
            setattr(parent, leaf, MXLinear(module, rules[hit][1], chunk, cache_weights))
            replaced.append((parent, leaf, module))
    cored, previous = [], None
    if not dry_run and any(core_of(hit) is not None for *_, hit in cores):
        register()
        previous = model.config._attn_implementation
        for _, module, hit in {id(m): (n, m, h) for n, m, h in cores if core_of(h) is not None}.values():
            module._mxq_core = core_of(hit)
            if vector["softmax"]:
                module._mxq_vector = vector["softmax"]
            cored.append(module)
        _set_attention(model, _CORE)
    normed = []
    if not dry_run:
        for (_, module), e in zip(norms, eps):
            module.forward = partial(_rmsnorm_forward, module, e, vector["rmsnorm"])
            normed.append(module)
    handle = Handle(model, table, replaced, core_table, cored, previous, vector, [n for n, _ in norms], normed)
    if dry_run:
        print(handle)
    return handle
