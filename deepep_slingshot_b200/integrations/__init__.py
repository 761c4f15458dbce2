"""Integrations with serving frameworks (SGLang-style normal-mode dispatcher)."""
