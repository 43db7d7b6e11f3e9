"""OpenAI- and Anthropic-compatible HTTP serving over the engine."""
