"""Core primitives: process groups, launch, hooks, precision."""
