"""mxq.nn — putting Schemes into a model.

    MXLinear(linear, scheme)     one nn.Linear computed through one Scheme (inference only)
    patch(model, rules)          a Scheme per layer name or type (first matching rule wins); (qk, pv) pairs route an
                                 attention module's core through attend
    is_attention                 a selector for the attention projections
    attend(q, k, v, mask, scale, qk, pv)   the attention core with Q·Kᵀ and P·V through two Schemes
"""
from ._attention import attend
from ._linear import MXLinear
from ._patch import is_attention, patch

__all__ = ["MXLinear", "patch", "is_attention", "attend"]
