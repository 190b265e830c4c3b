"""compiler subpackage."""
