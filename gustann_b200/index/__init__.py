"""Synthetic data and index construction for the search path."""
