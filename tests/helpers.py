"""Re-exports of conftest helpers for test modules."""
from conftest import from_bits, rel_err, to_bits  # noqa: F401
