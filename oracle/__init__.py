"""CPU oracle of PONNI's batched-inference path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
package, as the checker and the timed CPU baseline; libponni_b200 never calls it.
"""
