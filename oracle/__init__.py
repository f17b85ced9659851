"""CPU oracle of the reference's paged/varlen attention forward -- test infrastructure
only (tests/, __graft_entry__.smoke(), bench.py's CPU baseline); never imported by the
dvattn_b200 package."""
