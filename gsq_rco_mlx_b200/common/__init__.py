"""Evaluation of quantized models (reference src/gsq_rco/common)."""
