"""Test-only CPU oracle (see w4a16_oracle.py). Never imported by the shipped package."""
from .w4a16_oracle import *  # noqa: F401,F403
