"""CPU oracle of the Polar Switch hot path -- test infrastructure only.

Used by tests/, __graft_entry__.smoke() and the CPU-baseline leg of bench.py
as the checker or the timed CPU reference. The product package
(polar_switch) never imports anything from here.
"""
