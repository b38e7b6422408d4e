"""Test infrastructure: CPU restatements of the reference's scan path.

Nothing in the shipped package imports this; only tests, the smoke check and the
CPU-baseline arm of ``bench.py`` do.
"""
