"""Serving-engine adapters."""
