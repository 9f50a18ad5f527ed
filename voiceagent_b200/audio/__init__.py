"""Audio accounting, frontend and cross-request encoder packing."""
