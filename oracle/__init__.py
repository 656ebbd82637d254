"""CPU oracle of the attention forward path -- test infrastructure only.

Imported only by tests/, __graft_entry__.smoke() and bench.py's CPU baseline
and reference arm; never by the library (which has no CPU fallback).
"""
