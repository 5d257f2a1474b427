"""CPU oracle of the decode path: test infrastructure only (tests/, __graft_entry__.smoke(), bench.py's
CPU baseline). The product package rapier_b200 never imports it."""
