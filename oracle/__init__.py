"""CPU oracle for the fused linear + CE + entropy path (TEST INFRASTRUCTURE ONLY).

Imported only by tests/, __graft_entry__.smoke() and bench.py (cpu_baseline and --impl
reference legs). The product package never imports it. See reference_math.py.
"""
