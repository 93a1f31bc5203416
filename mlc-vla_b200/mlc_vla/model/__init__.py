"""Model definitions (the π0.5 backbone build is the only one on the hot path)."""
