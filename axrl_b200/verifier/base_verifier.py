"""Verifier interface: score a response against a reference answer."""

from __future__ import annotations


class BaseVerifier:
    def verify(self, response: str, answer: str) -> float:
        raise NotImplementedError
