"""Lowering recipes per target."""
