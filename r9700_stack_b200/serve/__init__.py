"""Serving front end: an asyncio engine wrapper, an OpenAI-compatible HTTP server, launchers and a
benchmark client (the role `vllm serve` + serve/*.sh + bench/harness.py play for the reference)."""
