"""Serving integrations: the engine seam (bridge, sessions, controls) and its configuration."""
