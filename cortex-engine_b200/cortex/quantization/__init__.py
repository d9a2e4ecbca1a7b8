"""Per-output-channel INT8 weight quantization (``cortex.quantization.calibrate``)."""
