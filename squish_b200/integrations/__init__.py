"""Integrations with other frameworks."""
