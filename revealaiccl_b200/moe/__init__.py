"""moe subpackage."""
