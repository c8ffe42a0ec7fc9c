"""Offline evidence analysis (CPU only)."""
