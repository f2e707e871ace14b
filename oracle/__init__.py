"""CPU oracle of the fused MoE operator -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py``
(plus ``bench.py --impl reference``) may import this package; the product library in
``fused-moe-yws_b200/`` never does. See ``fmoe_ref.py`` (PyTorch/C restatement of the
reference algorithm, parity pinned by ``tests/golden``) and ``fmoe_oracle.c``.
"""
from .fmoe_ref import (build, dequant_act, dequant_weight, moe_forward,  # noqa: F401
                       moe_forward_routed, plan, route, route_definition, route_margin,
                       sigmoid)
