from .runtime import MetalRuntime, PreparedKernel, Runtime  # noqa: F401
