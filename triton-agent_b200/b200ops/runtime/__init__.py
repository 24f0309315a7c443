"""ctypes binding of libb200ops.so and the torch-facing operator calls."""
