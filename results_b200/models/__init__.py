"""Synthetic model state_dicts of the shapes the reference measures."""
