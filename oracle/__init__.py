"""CPU oracle (test infrastructure): restatements of the reference's CPU path used as the checker.

Only the test suite, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may
import this package; the product package never does.
"""
