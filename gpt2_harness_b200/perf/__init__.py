"""perf subpackage."""
