"""Device-timed latency of the matmul_epilogue CUDA variant, CUDA events on
the launching stream."""

from b200ops.core.profiler import profile_kernel


def benchmark_matmul_epilogue(kernel_fn, inputs, warmup=20, repeat=100, flush_l2=False):
    return profile_kernel(kernel_fn, inputs, warmup=warmup, repeat=repeat, flush_l2=flush_l2)
