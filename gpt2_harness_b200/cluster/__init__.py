"""cluster subpackage."""
