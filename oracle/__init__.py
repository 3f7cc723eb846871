"""CPU oracle of the Flash-EKV LUT path — TEST INFRASTRUCTURE ONLY.

Imported by tests/, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
bench.py as the checker; the operator never imports it.
"""
