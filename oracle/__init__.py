"""Parity oracle of tilegen_b200 -- TEST INFRASTRUCTURE ONLY.

CPU restatement of TileGen's sparse kernels (``tg_oracle.c``), the recipe that compiles
it and the reference's own CPU code (``build.py``), and the ctypes front end
(``oracle.py``).  Imported only by ``tests/``, ``__graft_entry__.smoke()`` and the CPU
legs of ``bench.py``; the product path (``tilegen_b200``) never imports it.
"""
