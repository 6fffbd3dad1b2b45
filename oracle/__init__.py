"""CPU restatements of vidax's attention semantics -- test infrastructure only.

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU baseline and
reference arm; never by the vidax_b200 package.
"""
