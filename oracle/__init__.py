"""CPU oracle for breccia's hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in NumPy, the reference implementation of
``breccia.cast`` / ``dequantize`` / ``requantize`` / ``matmul``
(jvoltci/breccia v0.1.3, ``src/breccia/kernels/reference/`` and
``src/breccia/_formats.py``). It is the checker the parity tests compare the
CUDA kernels against, and the CPU baseline that ``bench.py`` times.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
``cpu_baseline`` / ``--impl reference`` legs may import it. The product
package ``breccia_b200`` never imports, calls or links it.

Parity is pinned: ``tests/golden/`` holds vectors produced by running the
reference itself (``tests/golden/make_golden.py``), and
``tests/test_oracle_golden.py`` checks this package against them bit for bit.
"""

from . import codec, cast  # noqa: F401
