"""Command line interface."""
