"""CPU oracle of the reference's joint-attention path — test and baseline infrastructure.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import
this package.  ``reference`` is the numpy restatement; ``cpu`` loads the C restatement
(``cpu_attention.c``, built by ``oracle/Makefile``).
"""
