"""CPU oracle for the Swin3D backbone block hot path.

TEST INFRASTRUCTURE ONLY. Nothing in the product package ``flash_aurora_b200`` imports this
package. It is imported by ``tests/``, by ``__graft_entry__.smoke()`` (as the checker) and by
``bench.py``'s CPU-baseline / ``--impl reference`` leg (as the timed CPU restatement of the
reference algorithm), and nowhere else.

Contents
--------
``oracle.layout``  numpy restatement of the window geometry, the fused cyclic shift + zero-pad
                   + 3D window partition and its inverse, and the shifted-window mask groups
                   (integer/index work, bit-exact).
``oracle.block``   torch-CPU FP32 restatement of AdaLN/FiLM, window attention (SDPA semantics
                   with the additive -100 Swin mask), the MLP, the Swin3D block, patch
                   merging/splitting and the U-net backbone forward.

Every function cites the upstream Flash-Aurora file:line it restates. The restatement is
pinned against fixtures produced by the upstream code itself (``tests/golden/make_golden.py``).
"""
