"""optim package."""
