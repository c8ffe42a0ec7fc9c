"""Fault-tolerance control plane: lighthouse, manager, transport, handoff."""
