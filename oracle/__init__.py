"""CPU oracle of the reference's LoRA hot path — test infrastructure only.

Used by tests/, ``__graft_entry__.smoke()`` (as the checker) and the CPU
baseline arm of bench.py. Never imported by the ``multi_lora_b200`` package.
Parity is pinned against golden vectors made from the reference's own code
(tests/golden/make_golden.py).
"""
