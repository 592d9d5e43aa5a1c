"""CPU oracle for the FusedSpikeBlock path -- test infrastructure only.

Imported by ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline /
reference arm of ``bench.py``; never by the product package.
"""
