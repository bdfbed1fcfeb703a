"""CUDA runtime layer: device context, caching allocator, streams and events."""
