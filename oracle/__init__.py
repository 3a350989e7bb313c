"""TEST INFRASTRUCTURE ONLY: the oracle for the B200 kernels.

Restatements of ducviet00/cpu-attention's algorithm for its three hot entry
points, used by ``tests/`` as the checker, by ``__graft_entry__.smoke()`` and by
``bench.py``'s CPU-baseline leg. Nothing in the product path
(``cpu-attention_b200/``) imports, links or calls anything here.

* ``attention_f64``: the reference's float64 eager oracle and its gates
  (``tests/reference.py:7-40`` of the reference), restated in numpy.
* ``paged``: the reference's paged-cache byte layout and ``reshape_and_cache``
  scatter (``paged_attn.mojo:58-176``), restated in numpy (bit-exact checks).
* ``cpu``: ctypes access to ``ca_oracle.c``, the C restatement of the
  reference's CPU kernel numerics (decode, store, flash) with OpenMP -- the
  timed CPU baseline and the north-star tolerance reference.

Parity pin: the reference's Mojo kernel cannot be built here (no Mojo
toolchain), so ``attention_f64`` and ``cpu`` are pinned against golden vectors
that the reference's own float64 oracle produced (``tests/golden``).
"""
