"""Utilities: clock sampling, device timing, logging."""
