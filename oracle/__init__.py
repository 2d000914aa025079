"""Test infrastructure: the CPU oracle and the reference-PTX runner for irptx-b200.

Nothing here is on the product path. Only tests/, __graft_entry__.smoke() and bench.py's
baseline legs import it, and only as the checker: the product (irptx_b200, libirx.so) never
imports, links or runs anything under oracle/.
"""
