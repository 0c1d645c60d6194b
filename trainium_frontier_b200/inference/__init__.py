"""inference package."""
