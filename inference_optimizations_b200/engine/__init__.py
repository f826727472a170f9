"""engine package."""
