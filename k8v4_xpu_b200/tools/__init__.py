"""Offline tools: GPTQ bake, checkpoint assembly and verification, random-init checkpoints."""
