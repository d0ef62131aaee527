"""CPU oracle for the paged KV-cache path — TEST INFRASTRUCTURE ONLY.

Restatements of the reference algorithms (NumPy), used by tests/, by
__graft_entry__.smoke() as the checker, and by bench.py's CPU-baseline leg.
The product package (synapcore_b200) never imports this package.
"""
