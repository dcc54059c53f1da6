"""megamoe: B200-native (sm_100a) routed-MoE chain behind the reference's step API.

``RoutedMoE`` binds one MoE layer's MXFP4 weights; the stateless ops
(``router_gemv``, ``gate_topk``, ``route``, ``finalize``) mirror the reference's
individual kernels. All compute runs in libmegamoe.so (hand-written CUDA for
sm_100a); there is no CPU path.
"""

from .moe import (  # noqa: F401
    RoutedMoE,
    finalize,
    finalize_partial,
    gate_topk,
    route,
    route_words,
    router_gemv,
)
from .comm import PeerAllReduce  # noqa: F401
from .stack import MoEStack  # noqa: F401

__all__ = ["MoEStack", "PeerAllReduce", "RoutedMoE", "finalize", "finalize_partial", "gate_topk", "route", "route_words", "router_gemv"]
