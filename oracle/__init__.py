"""CPU oracle of the chess-engine-4 forward path — TEST INFRASTRUCTURE ONLY.

Imported only by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg, as the
checker. The product path (libce4b200 and the ce4b200 package) never imports it.
"""
