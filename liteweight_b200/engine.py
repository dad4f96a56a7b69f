"""Native decode engine (the fused decode kernels are not built yet)."""


def supports(model) -> bool:
    return False
