"""Adapters between the engine and the reference's integration points."""
