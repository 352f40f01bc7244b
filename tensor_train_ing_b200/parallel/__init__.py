"""Data-parallel runtime: process groups, gradient arenas and the collective paths."""
