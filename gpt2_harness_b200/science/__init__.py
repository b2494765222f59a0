"""science subpackage."""
