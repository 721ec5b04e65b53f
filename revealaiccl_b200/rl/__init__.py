"""rl subpackage."""
