"""Offline conversion tools: chat JSONL -> manifest v1, HF hybrid -> Lightning PTH, TimeMix splice."""
