"""scheduling subpackage."""
