"""kv package."""
