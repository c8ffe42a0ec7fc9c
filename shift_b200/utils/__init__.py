"""Shared utilities: digests, JSONL events, timing."""
