"""server package."""
