"""Launcher: resolve a settings directory into the server command."""
