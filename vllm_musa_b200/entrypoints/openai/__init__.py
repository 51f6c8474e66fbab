"""OpenAI-compatible HTTP server."""
