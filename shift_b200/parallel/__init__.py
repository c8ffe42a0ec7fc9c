"""Flat parameter storage, parallel layouts and collectives."""
