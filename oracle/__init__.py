"""Test infrastructure: the CPU oracle (a float64 restatement of the reference's op
semantics). Imported only by tests/, ``__graft_entry__.smoke()`` and bench.py's CPU
baseline; never by the product path."""
