"""Runnable examples: the vLLM KV connector on a real vLLM engine (and a
sweep over restore sizes), a vLLM environment probe, one generic transfer
intent through the public client, and slot-adapter entry points."""
