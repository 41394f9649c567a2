"""Quality evaluation drivers (GSM8K exact match, MT-Bench generation + LLM judge)."""
