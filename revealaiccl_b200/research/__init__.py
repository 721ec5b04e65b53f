"""research subpackage."""
