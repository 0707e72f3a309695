"""Error type of the operator API (the reference's ModelSharpException)."""
from __future__ import annotations


class ModelSharpException(Exception):
    """Raised for invalid graphs / inputs and backend failures; `status` is the C-ABI code."""

    def __init__(self, message: str, status: int | None = None):
        super().__init__(message)
        self.status = status
