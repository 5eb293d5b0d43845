"""Test infrastructure: the CPU/GPU oracle for the Wan2.1 DiT block's non-attention half.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm may import
this package, and only as the checker. The product (coda-wan-dit_b200/) never imports it.

Parity anchor: the reference (Owen718/CODA-Wan-DiT) ships no tests or fixtures and its
GEMM arithmetic lives in an absent third-party package (coda-kernels `rapier`, unpinned),
so parity is pinned against golden vectors produced by running the reference's OWN Triton
aux kernels and table builder (coda_wan/wan_coda_kernels.py) on CPU through Triton's
interpreter (tests/golden/make_golden.py), plus the reference's published known answers
(RoPE table bytes, GELU constants, partial layout). The stock-Wan block/model math itself
(upstream Wan2.1 @ 9737cba9, not installed) is restated from the formulas in the
reference's docs/report.md:37-43 and docs/walkthrough.md:27-32; the non-block parts of the
model are marked "unverified vs upstream".
"""
