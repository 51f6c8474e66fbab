"""User entry points: offline ``LLM`` API, OpenAI-compatible server, CLI."""
