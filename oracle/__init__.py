"""CPU oracle for the MoE decode hot path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this package, and only as
the checker or the timed CPU baseline; the product (``joule_b200``) never
imports, loads or calls anything here.

Contents
  q4.py       numpy restatement of the reference's Q4 quantiser/dequantiser
  restate.py  ctypes front end of libjoule_oracle.so, this repo's C
              restatement of the reference's MoE layer (joule_oracle.c)
  ref.py      ctypes front end of _ref/libjoule_ref.so, the reference's own
              decode_kernel.c compiled unmodified (Makefile target ``ref``)
  layer.py    a synthetic Q4 MoE layer (seeded) in the reference's layout
"""
