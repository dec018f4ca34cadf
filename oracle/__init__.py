"""CPU oracle for the routed-expert NVFP4 (W4A16) MoE layer.

TEST INFRASTRUCTURE ONLY. Nothing in the shipped package imports this directory: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg (and its ``--impl reference`` arm) may use it, and
only as the checker or as the timed CPU baseline, never as the thing measured on the GPU.

Each module restates one piece of the reference's algorithm in plain numpy/torch-CPU code and cites the reference
file:line it follows (paths relative to the reference project; ``vllm/...`` paths point into vLLM 0.22.0's Python
sources):

- ``nvfp4``        E2M1 / E4M3 decoding and the per-expert dequantisation (bench/moek/problem.py:17-38).
- ``marlin_scales`` vLLM's Marlin scale preparation for NVFP4 (vllm/.../marlin_utils.py:296-316,
                   vllm/.../marlin_utils_fp4.py:30-146,355-386).
- ``scale_codec``  the kit's lossless packed-scale codec and item tiling (files/mbx_moek.py:61-172).
- ``align``        moe_align_block_size's sort-and-pad contract (vllm/.../moe_align_block_size.py:11-103).
- ``moe_ref``      the fp32 dequantise-then-matmul layer (bench/moek/problem.py:51-67) plus the kit kernel's
                   rounding points (files/mbx_moek.cu:143-148,616-647,797-833; files/mbx_moek.py:284-289).

Parity pins: ``tests/golden/make_golden.py`` runs the reference's own Python (files/mbx_moek.py's codec,
bench/moek/problem.py's ``reference``, vLLM's scale helpers) in the build container and stores the results as
fixtures under ``tests/golden/``; ``tests/test_oracle_golden.py`` checks every module here against them.
moe_align_block_size's compiled kernel cannot run without a GPU; it is pinned by its docstring example only.
"""
