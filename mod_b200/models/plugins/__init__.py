"""Model plugins: one package per model, each with a plugin_manifest.json."""
