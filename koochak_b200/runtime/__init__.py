"""Parts of ``training_loop``: settings, the gradient gate, checkpoint collection and resume."""
