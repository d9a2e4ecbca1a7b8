"""B200 kernels behind the reference's ``cortex.kernels`` API."""
