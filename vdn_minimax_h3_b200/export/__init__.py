"""Publishing a checkpoint as a self-contained model component (one flattened modeling
file + config.json pointing back at the checkpoint's tensors)."""
