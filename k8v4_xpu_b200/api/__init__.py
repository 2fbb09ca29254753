"""OpenAI-compatible serving: tokenizer, engine driver, HTTP server, metrics."""
