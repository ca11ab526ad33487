"""CPU oracle of vk-compute's decode path -- test infrastructure only.

Imported by tests/, the smoke check and the CPU-baseline leg of bench.py as
the checker; the product never imports it.
"""
