"""Node supervisor and in-box cluster controller."""
