"""CPU oracle for the KV block store (test infrastructure only).

`oracle.kvs_oracle` wraps the C restatement in kvs_oracle.c. Only the tests, the smoke
check and bench.py's CPU-baseline leg use it, and only as the checker or the timed CPU
baseline; the product in tt-infinity_b200/ never imports it.
"""
