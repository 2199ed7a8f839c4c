"""vLLM integration: platform class, attention backend, hooks, config policy."""
