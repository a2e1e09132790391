"""CPU oracle of the attention hot paths (test infrastructure only).

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg;
never by the attnkernels package.
"""
