"""formats subpackage."""
