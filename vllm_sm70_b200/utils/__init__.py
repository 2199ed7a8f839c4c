"""Logging, launch accounting and timing helpers."""
