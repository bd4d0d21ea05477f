"""Drop-in for profiling/int4_batched_gemm_v2.py (cache-barrier):
quantize_weights_int4_kpacked (:125-137), batched_int4_gemm (:239-260) and the
kernel_batched_w4a16_v3 launch object (:140-236), backed by libcb200's sm_100a
W4A16 kernel. The v2 file's K-packing is the same as bench_l2_barrier's."""

try:
    from . import _bootstrap  # noqa: F401
    from .bench_l2_barrier import _W4A16KernelLauncher, batched_int4_gemm, quantize_weights_int4
except ImportError:
    import _bootstrap  # noqa: F401
    from bench_l2_barrier import _W4A16KernelLauncher, batched_int4_gemm, quantize_weights_int4

quantize_weights_int4_kpacked = quantize_weights_int4
kernel_batched_w4a16_v3 = _W4A16KernelLauncher("kernel_batched_w4a16_v3")

__all__ = ["quantize_weights_int4_kpacked", "batched_int4_gemm", "kernel_batched_w4a16_v3"]
