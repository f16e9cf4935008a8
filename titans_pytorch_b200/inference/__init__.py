"""inference subpackage."""
