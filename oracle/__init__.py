"""CPU oracle for the quantized-weight hot path -- TEST INFRASTRUCTURE ONLY.

This package is a numpy restatement of the reference's algorithms for the
hot path (thedracle/deepseek-v41-mlx):

* ``formats``   -- deepseek_v41_mlx/dequant.py:24-84 (fp8 e4m3 / fp4 e2m1 /
                   ue8m0 decode) and the MLX affine group format
                   (deepseek_v41_mlx/convert.py:156-175, engram.py:206-223).
* ``act_quant`` -- upstream act_quant, docs/reference/kernel.py:40-124 as
                   transcribed by tests/kernel_stub.py:26-63.
* ``linear``    -- dequant-then-matmul products (the a16 form of upstream
                   linear(), docs/reference/model.py:181-207) and the MLX
                   quantized matmul.
* ``moe``       -- deepseek_v41_mlx/moe.py:30-112 (port semantics) and the
                   upstream MoE of docs/reference/model.py:792-904.
* ``engram``    -- deepseek_v41_mlx/engram.py:35-203 and upstream
                   ParallelEngramEmbedding (docs/reference/model.py:296-325).

Who may use it: only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``
(its ``cpu_baseline`` leg and its ``--impl reference`` arm), and only as the
checker / the timed CPU baseline.  The product package never imports it.

Parity pinning: the reference's own MLX code cannot run here (mlx is not
installable offline), so the oracle is pinned against golden vectors made by
``tests/golden/make_golden.py`` from the parts of the reference that do run on
CPU: the torch halves of tests/test_parity.py:348-387, tests/kernel_stub.py
act_quant, the port's numpy EngramHasher, upstream NgramHashState, Gate and
Expert.  The MLX affine quantized-matmul numerics are not pinned by any
reference test (only finiteness, tests/test_parity.py:583-586); that row is
"parity unpinned" and the oracle's definition is stated in ``formats``.
"""
