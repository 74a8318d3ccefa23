"""Parallelism: device meshes, FSDP2 / HSDP / TP application, pipeline
schedule helpers, and device timing across ranks."""
