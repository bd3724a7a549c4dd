"""CPU checkers for the sparse-decode path (test infrastructure only).

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of ``bench.py``
import this package.  The product library never links or calls it.
"""
