"""Serving-side batch assembly for the B200 forward (cortex/serve in the reference)."""
