"""sb200 — host side of the B200 hot path (router + ternary experts).

``sb200._lib`` binds libspectral_b200.so; ``sb200.router`` and
``sb200.ternary`` wrap its handles for torch tensors; ``sb200.synth`` holds
the seeded workload recipes.  The drop-in modules that mirror the reference's
own import names (``bvh_router``, ``ternary_expert_ext``,
``ternary_expert_ext_bridge``, ``spectral_ai``) sit next to this package.
"""

__all__ = ["synth"]
