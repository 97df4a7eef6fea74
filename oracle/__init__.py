"""CPU oracle for the sampling path (test infrastructure only).

Importable by the tests, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py``; never by the product package ``neuraval_b200``.
"""
