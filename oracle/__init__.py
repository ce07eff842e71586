"""CPU oracle for the piecewise-linear embedding path (test infrastructure).

Nothing in the product package imports this directory. Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` use it,
always as the checker or as the timed CPU stand-in, never as the product.
"""
