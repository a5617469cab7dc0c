"""CPU oracle of the chunked Gated DeltaNet forward (test infrastructure only).

Imported only by tests/, __graft_entry__.smoke() and the CPU-baseline legs of
bench.py, always as the checker; the gdn_b200 product path never uses it.
"""
