"""spectral_ai — package facade of the B200 hot path.

Same names as the reference facade (spectral_ai/__init__.py:53-70) for the
parts this repository provides: BVHRouter, BranchSpecificBVHRouter (raises:
not on the hot path), RouterConfig, RoutingResult, HybridBVHRouter; plus the
B200 MoE layer pieces.  ExpertLRUCache (host-side expert caching) is not
provided: the experts stay resident in HBM.
"""

import sys
from pathlib import Path

_pkg_dir = Path(__file__).resolve().parent.parent
if str(_pkg_dir) not in sys.path:
    sys.path.insert(0, str(_pkg_dir))

from bvh_router import BVHRouter, BranchSpecificBVHRouter, RouterConfig, RoutingResult  # noqa: E402
from bvh_router_bridge import HybridBVHRouter  # noqa: E402
from sb200.moe import BVHMoELayer  # noqa: E402
from sb200.ternary import TernaryExperts  # noqa: E402

__all__ = [
    "BVHRouter",
    "BranchSpecificBVHRouter",
    "RouterConfig",
    "RoutingResult",
    "HybridBVHRouter",
    "BVHMoELayer",
    "TernaryExperts",
]

__version__ = "0.1.0"
