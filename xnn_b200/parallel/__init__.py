"""Distribution: process-group helpers, data-parallel gradient sync, spatial domain decomposition."""
