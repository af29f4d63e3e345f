"""Sampling and tokenizer helpers."""
