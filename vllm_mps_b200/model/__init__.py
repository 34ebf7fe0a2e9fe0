"""Token sampling."""
