"""Step packing, MuWorker and the engines."""
