"""Prompt-side helpers (compression)."""
