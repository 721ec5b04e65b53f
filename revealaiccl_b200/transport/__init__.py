"""transport subpackage."""
