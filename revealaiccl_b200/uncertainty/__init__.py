"""uncertainty subpackage."""
