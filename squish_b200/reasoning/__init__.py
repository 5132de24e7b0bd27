"""Answer aggregation across sampled reasoning chains."""
