"""Harness that runs the unmodified reference implementation for the benchmark's reference arm."""
