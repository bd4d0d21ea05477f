"""Drop-in for profiling/int4_batched_gemm.py (cache-barrier): the MLA
reconstruction batched INT4 BMM API (quantize_weights_int4 :212-229,
batched_int4_gemm :232-265, kernel_batched_w4a16_simple :130-205), backed by
libcb200's sm_100a W4A16 kernel. See bench_l2_barrier.py in this directory."""

try:
    from . import _bootstrap  # noqa: F401
    from .bench_l2_barrier import (_W4A16KernelLauncher, batched_int4_gemm,  # noqa: F401
                                   quantize_weights_int4)
except ImportError:
    import _bootstrap  # noqa: F401
    from bench_l2_barrier import _W4A16KernelLauncher, batched_int4_gemm, quantize_weights_int4  # noqa: F401

kernel_batched_w4a16_simple = _W4A16KernelLauncher("kernel_batched_w4a16_simple")
kernel_batched_w4a16_gemm = _W4A16KernelLauncher("kernel_batched_w4a16_gemm")

# MLA reconstruction shapes used by the reference benches (:272-275).
H = 128
D_NOPE = 128
KV_LORA = 512
D_V = 128
