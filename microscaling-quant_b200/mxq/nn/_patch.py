"""patch(model, rules): which Scheme each nn.Linear (and each attention core) of a model runs through
(mxq/nn/_patch.py:123-287 of the reference; same API, rules, checks, messages and printed table).

    rules = [("lm_head", None),                        # a layer name, * wildcards; None leaves the layer as it is
             ("*.mlp.down_proj", FP6),                 # a Scheme
             (is_attention, None),                     # a function (name, module, parent) -> bool
             (nn.Linear, FP8),                         # a layer type
             ("model.layers.*.self_attn", (QK, PV))]   # a pair of Schemes: that attention module's core
    handle = patch(model, rules)                       # the first rule that matches a layer decides it
    handle.revert()                                    # everything patch changed, undone
    patch(model, rules, dry_run=True)                  # print the table, change nothing

How it works here. `_Survey` walks the model once, keeping every name under which a module is reachable, and lists
the Linear layers and the attention modules (those holding q_proj and k_proj) with their parents. `_decide` gives
each its rule and checks the choice as a whole: every rule must choose something, an attribute reached under
several names must get one rule, an attention module reached under several names too. Before the model is
touched, every Scheme runs once on a tiny matmul (and every core on a tiny attention), so a bad schedule or format
fails here. The changes are then made one by one, each recording how to undo itself in the Handle's log;
`revert` plays the log backwards.

vector="bf16" (or {"softmax": ..., "rmsnorm": ...}) rounds the vector ops' steps to bf16: softmax runs in attend
(attention modules without a core rule get the EXACT core, since sdpa's fused kernel has no step to round), and
every *RMSNorm forward is replaced after a check that the unrounded replacement reproduces the module's own output
bit for bit.
"""
from dataclasses import dataclass
from fnmatch import fnmatchcase
from functools import partial
from typing import Callable, Dict, List, Optional, Sequence, Tuple, Union

import torch
from torch import nn

from ..scheme import Scheme
from ._attention import NAME as _CORE, attend, register
from ._linear import MXLinear
from ._vector import EXACT, resolve, rmsnorm

__all__ = ["patch", "is_attention", "Handle"]

Selector = Union[str, type, Callable[[str, nn.Module, nn.Module], bool]]
Rule = Tuple[Selector, Union[None, Scheme, Tuple[Scheme, Scheme]]]


def is_attention(name: str, module: nn.Module, parent: nn.Module) -> bool:
    """Is this Linear one of an attention module's projections? True when its parent holds both q_proj and k_proj
    (the test MXQuant's eval_complete.py uses, so a rule list written with it keeps MXQuant's layer set)."""
    return _attention_module(parent)


def _attention_module(module: nn.Module) -> bool:
    return hasattr(module, "q_proj") and hasattr(module, "k_proj")


def _core_pair(value) -> bool:
    """A rule value that chooses an attention core: (qk Scheme, pv Scheme)."""
    return isinstance(value, tuple) and len(value) == 2 and all(isinstance(s, Scheme) for s in value)


def _selects(selector: Selector, name: str, module: nn.Module, parent: nn.Module) -> bool:
    if isinstance(selector, type):
        return isinstance(module, selector)
    if isinstance(selector, str):
        return fnmatchcase(name, selector)
    return bool(selector(name, module, parent))


# -------------------------------------------------------------------------------------------- survey
@dataclass
class _Seen:
    """One module under one of its names; `rule` is the index of the rule that chose it (None: no rule)."""
    name: str
    module: nn.Module
    parent: nn.Module
    rule: Optional[int] = None

    @property
    def attr(self) -> str:
        return self.name.rsplit(".", 1)[-1]


class _Survey:
    """Every name under which each module is reachable (a module held twice is listed twice), split into the
    Linear layers, the attention modules and the RMSNorm modules."""

    def __init__(self, model: nn.Module):
        named = dict()
        order = []
        for name, module in model.named_modules(remove_duplicate=False):
            named[name] = module
            order.append((name, module))
        def parent(name):
            return named[name.rsplit(".", 1)[0] if "." in name else ""]
        self.linears = [_Seen(n, m, parent(n)) for n, m in order if n and isinstance(m, nn.Linear)]
        self.attention = [_Seen(n, m, parent(n)) for n, m in order if n and _attention_module(m)]
        norms: Dict[int, Tuple[str, nn.Module]] = {}
        for n, m in order:
            if n and type(m).__name__.endswith("RMSNorm") and id(m) not in norms:
                norms[id(m)] = (n, m)
        self.norms = list(norms.values())


def _decide(rules: Sequence[Rule], survey: _Survey) -> None:
    """Give every surveyed Linear and attention module its rule (first match of its kind), then refuse a choice
    that cannot be carried out as asked."""
    for i, rule in enumerate(rules):
        if len(rule) != 2 or not (rule[1] is None or isinstance(rule[1], Scheme) or _core_pair(rule[1])):
            raise ValueError(f"rule {i} must be (selector, Scheme or None or (qk Scheme, pv Scheme)), got {rule!r}")
    kinds = {False: [], True: []}                          # is a core rule -> rule indices, in order
    for i, (_, value) in enumerate(rules):
        kinds[_core_pair(value)].append(i)
    for seen, candidates in ((survey.linears, kinds[False]), (survey.attention, kinds[True])):
        for s in seen:
            s.rule = next((i for i in candidates if _selects(rules[i][0], s.name, s.module, s.parent)), None)

    idle = [i for i in kinds[False] if i not in {s.rule for s in survey.linears}]
    if idle:
        raise ValueError(f"rules {idle} choose no Linear layer (misspelt, or hidden behind an earlier rule): "
                         f"{[rules[i][0] for i in idle]}")
    idle = [i for i in kinds[True] if i not in {s.rule for s in survey.attention}]
    if idle:
        raise ValueError(f"rules {idle} choose no attention module (one holding q_proj and k_proj): "
                         f"{[rules[i][0] for i in idle]}")
    # an attention module chosen under one of its names must be chosen the same way under all of them
    by_module: Dict[int, List[_Seen]] = {}
    for s in survey.attention:
        by_module.setdefault(id(s.module), []).append(s)
    for group in by_module.values():
        if any(s.rule is not None for s in group) and len({s.rule for s in group}) > 1:
            raise ValueError(f"{[s.name for s in group]} are the same attention module but match different rules; "
                             "one of them has to go")
    # a Linear runs from an attribute of its parent; every name reaching that attribute must agree
    for group in _sites(survey.linears).values():
        if len({s.rule for s in group}) > 1:
            raise ValueError(f"{[s.name for s in group]} are the same layer but match different rules "
                             f"{[s.rule for s in group]}; one of them has to go")


def _sites(linears: List[_Seen]) -> Dict[Tuple[int, str], List[_Seen]]:
    """The Linear layers grouped by the attribute they are held in: (id of parent, attribute name)."""
    sites: Dict[Tuple[int, str], List[_Seen]] = {}
    for s in linears:
        sites.setdefault((id(s.parent), s.attr), []).append(s)
    return sites


# ------------------------------------------------------------------------------------------ dry runs
def _try_scheme(scheme: Scheme) -> None:
    """One tiny matmul: two whole LUT groups of columns, three blocks of contraction (so the scale check runs)."""
    g = torch.Generator().manual_seed(0)
    cols, depth = 2 * scheme.rows, 3 * scheme.block_size
    scheme.matmul(torch.randn(depth, cols, generator=g), torch.randn(depth, cols, generator=g))


def _try_core(qk: Scheme, pv: Scheme) -> None:
    """One tiny grouped-query attention: whole key blocks and whole LUT groups."""
    g = torch.Generator().manual_seed(0)
    tokens = 2 * max(qk.block_size, pv.block_size) * max(qk.rows, pv.rows)
    q, k, v = (torch.randn(1, heads, tokens, 32, generator=g) for heads in (2, 1, 1))
    attend(q, k, v, None, 32 ** -0.5, qk, pv)


def _norm_eps(name: str, module: nn.Module) -> float:
    """The module's epsilon, after checking that rmsnorm(·, precision=None) is its forward, bit for bit."""
    weight = getattr(module, "weight", None)
    if not isinstance(weight, torch.Tensor) or weight.ndim != 1:
        raise ValueError(f"{name} ({type(module).__name__}): no 1-D weight, not the RMSNorm mxq knows")
    eps = next((getattr(module, a) for a in ("variance_epsilon", "eps") if isinstance(getattr(module, a, None), float)),
               None)
    if eps is None:
        raise ValueError(f"{type(module).__name__}: no float variance_epsilon or eps attribute")
    probe = torch.randn(3, weight.shape[0], generator=torch.Generator().manual_seed(0)) * 3
    probe = probe.to(device=weight.device, dtype=weight.dtype)
    with torch.no_grad():
        own, mine = module(probe), rmsnorm(probe, weight, eps, None)
    if own.dtype != mine.dtype or not torch.equal(own, mine):
        raise ValueError(f"{name} ({type(module).__name__}) does not compute weight · x / sqrt(mean(x²) + eps) the way "
                         "transformers' LlamaRMSNorm does; vector rmsnorm cannot replace it")
    return eps


def _norm_forward(module: nn.Module, eps: float, precision: str, x: torch.Tensor) -> torch.Tensor:
    return rmsnorm(x, module.weight, eps, precision)


def _attention_impl(model: nn.Module, name: str) -> None:
    if hasattr(model, "set_attn_implementation"):
        model.set_attn_implementation(name)
    else:
        model.config._attn_implementation = name


# -------------------------------------------------------------------------------------------- handle
class Handle:
    """What patch did. `table`: one row per Linear name, (name, in, out, rule index or None, Scheme name or None);
    `cores`: one row per attention module name, (name, rule index or None, (qk name, pv name) or None); `vector`:
    the resolved vector setting; `norms`: the RMSNorm modules whose forward was replaced. `revert()` undoes every
    change, last first."""

    def __init__(self, table, cores, vector, norms):
        self.table, self.cores, self.vector, self.norms = table, cores, vector, norms
        self._undo: List[Callable[[], None]] = []

    def _did(self, undo: Callable[[], None]) -> None:
        self._undo.append(undo)

    def revert(self) -> None:
        while self._undo:
            self._undo.pop()()

    def __str__(self) -> str:
        w = max([5] + [len(r[0]) for r in self.table] + [len(r[0]) for r in self.cores])
        mark = lambda rule: "-" if rule is None else rule                     # noqa: E731
        out = [f"{'layer':{w}s}  {'in':>6s} {'out':>6s}  rule  scheme"]
        for name, fan_in, fan_out, rule, scheme in self.table:
            what = "no rule" if rule is None else (scheme or "left as is")
            out.append(f"{name:{w}s}  {fan_in:6d} {fan_out:6d}  {mark(rule):>4}  {what}")
        if any(names is not None for *_, names in self.cores):
            out.append(f"{'attention core':{w}s}  {'':13s}  rule  Q·Kᵀ, P·V")
            for name, rule, names in self.cores:
                what = "sdpa (no rule)" if names is None else ", ".join(names)
                if rule is None and names is not None:
                    what += "  (vector softmax)"
                out.append(f"{name:{w}s}  {'':13s}  {mark(rule):>4}  {what}")
        if any(self.vector.values()):
            count = {"softmax": sum(names is not None for *_, names in self.cores), "rmsnorm": len(self.norms)}
            parts = []
            for op, precision in self.vector.items():
                parts.append(f"{op} {precision or 'as transformers'}" + (f" ({count[op]} modules)" if precision else ""))
            out.append("vector  " + ", ".join(parts))
        return "\n".join(out)


# --------------------------------------------------------------------------------------------- patch
def patch(model: nn.Module, rules: Sequence[Rule], chunk: Optional[int] = None, dry_run: bool = False,
          cache_weights: bool = True, vector=None) -> Handle:
    """Route the model's Linear layers (and attention cores) through the Schemes the rules choose; see the module
    docstring. Returns a Handle (printed, with nothing changed, when dry_run)."""
    vector = resolve(vector)
    survey = _Survey(model)
    _decide(rules, survey)
    if vector["softmax"] and not survey.attention:
        raise ValueError("vector softmax: the model has no attention module (one holding q_proj and k_proj)")
    norms = survey.norms if vector["rmsnorm"] else []
    if vector["rmsnorm"] and not norms:
        raise ValueError("vector rmsnorm: the model has no module whose class name ends in RMSNorm")

    def core(rule):                                          # the (qk, pv) an attention module runs; None: sdpa
        if rule is not None:
            return rules[rule][1]
        return (EXACT, EXACT) if vector["softmax"] else None

    # everything that could fail runs before the model is touched
    for selector, value in rules:
        if isinstance(value, Scheme):
            _try_scheme(value)
    for selector, value in rules:
        if _core_pair(value):
            _try_core(*value)
    if vector["softmax"] and any(s.rule is None for s in survey.attention):
        _try_core(EXACT, EXACT)
    eps = [_norm_eps(n, m) for n, m in norms]

    def scheme_name(rule):
        return None if rule is None or rules[rule][1] is None else rules[rule][1].name

    table = [(s.name, s.module.in_features, s.module.out_features, s.rule, scheme_name(s.rule))
             for s in survey.linears]
    cores = [(s.name, s.rule, None if core(s.rule) is None else tuple(x.name for x in core(s.rule)))
             for s in survey.attention]
    handle = Handle(table, cores, vector, [n for n, _ in norms])
    if dry_run:
        print(handle)
        return handle

    for group in _sites(survey.linears).values():
        s = group[0]
        if s.rule is None or rules[s.rule][1] is None:
            continue
        setattr(s.parent, s.attr, MXLinear(s.module, rules[s.rule][1], chunk, cache_weights))
        handle._did(partial(setattr, s.parent, s.attr, s.module))

    routed = {}                                              # id -> (module, core), one entry per module
    for s in survey.attention:
        if core(s.rule) is not None:
            routed[id(s.module)] = (s.module, core(s.rule))
    if routed:
        register()
        before = model.config._attn_implementation
        for module, pair in routed.values():
            module._mxq_core = pair
            if vector["softmax"]:
                module._mxq_vector = vector["softmax"]
            handle._did(partial(_drop_core, module))
        _attention_impl(model, _CORE)
        handle._did(partial(_attention_impl, model, before))

    for (name, module), e in zip(norms, eps):
        module.forward = partial(_norm_forward, module, e, vector["rmsnorm"])
        handle._did(partial(delattr, module, "forward"))     # the class's own forward again
    return handle


def _drop_core(module: nn.Module) -> None:
    del module._mxq_core
    if hasattr(module, "_mxq_vector"):
        del module._mxq_vector
