"""launcher subpackage."""
