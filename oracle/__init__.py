"""CPU oracle for the strict int8 ECO training path (test infrastructure only).

This package restates, in numpy and plain Python, the integer algorithms of
``ecoint8`` v0.4.9 (``ecoint8/fixedpoint.py``, ``ecoint8/strict/ilayer.py``,
``ecoint8/strict/iopt.py``) and the fp32 algorithm of the Triton optimizer
(``ecoint8/triton_kernels.py``).  Each function cites the reference file:line it
follows.  It is the checker: only the test suite, ``__graft_entry__.smoke()``
and the CPU-baseline leg of ``bench.py`` may import it.  The CUDA library never
calls into it, and the product path raises when the CUDA extension is missing.

Parity pins: the fixtures under ``tests/golden/`` were produced by running the
reference itself (``tests/golden/make_golden.py``) and the oracle is checked
against every one of them by ``tests/test_oracle_golden.py``.
"""
