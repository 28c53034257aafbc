"""Runnable examples of the public API."""
