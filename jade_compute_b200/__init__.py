"""jade_compute_b200: B200-native (sm_100a) backend for Jade Compute's
KernelSpec -> compile -> ordered-batch execute hot path.

The product is the C-ABI library ``lib/libjade_runtime.so`` (declared in
``include/jade_runtime.h``); this package is its Python host mirror.
"""
from .runtime import (Buffer, Execution, JadeError, Kernel, Runtime, bf16_to_f32, canonical, comm_init_all,
                      comm_unique_id, device_count, emit, f32_to_bf16, lib, library_path, spec_bindings, spec_launch,
                      spec_validate, spec_validate_bindings)

__all__ = ["Buffer", "Execution", "JadeError", "Kernel", "Runtime", "bf16_to_f32", "canonical", "comm_init_all",
           "comm_unique_id", "device_count", "emit", "f32_to_bf16", "lib", "library_path", "spec_bindings",
           "spec_launch", "spec_validate", "spec_validate_bindings"]
