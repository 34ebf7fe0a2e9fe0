"""KV-cache pools: the device pool and the pinned-host swap space."""
