"""Drop-in replacements for the cache-barrier reference's quantized-GEMM modules.

Put this directory first on ``sys.path`` (before the reference's ``profiling/``,
``profiling/w8a8/`` and ``kernels/``) and the reference's harnesses import
``bench_l2_barrier``, ``int4_batched_gemm``, ``int4_batched_gemm_v2``,
``w8a8_bmm`` and ``triton_gemm`` from here: same names, same arguments, backed by
the sm_100a kernels of ``libcb200.so``.
"""
