"""CPU oracle for the decoder-engine path: test infrastructure, never the product.

Importable only from ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline / reference arm.
"""
