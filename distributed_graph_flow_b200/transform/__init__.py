"""Graph transforms used to prepare sampler inputs."""
