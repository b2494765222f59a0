"""Native (sm_100a) operators: thin validated wrappers over ``gpt2_harness_b200._C``."""

from gpt2_harness_b200.ops import native  # noqa: F401
from gpt2_harness_b200.ops.native import available, check_errors, lib  # noqa: F401
