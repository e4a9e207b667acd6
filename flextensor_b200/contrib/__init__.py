"""Integrations with serving / pipeline frameworks (imported on demand)."""
