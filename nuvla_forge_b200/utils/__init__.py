"""Utilities: environment description, hardware probe, fault injection helpers, watchdog."""
