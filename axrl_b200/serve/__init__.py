"""Standalone rollout/teacher servers and their HTTP router."""
