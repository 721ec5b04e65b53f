"""traffic subpackage."""
