"""Developer tooling: A/B switches between implementations and hot swaps between engine steps."""
