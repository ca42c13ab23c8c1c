"""tcgen05 block-scaled MXFP8 GEMM (placeholder until the kernel lands)."""


def applies(*args, **kwargs) -> bool:
    return False
