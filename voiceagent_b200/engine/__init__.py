"""Engine layer: request state, block manager, scheduler, runners and AsrEngine."""
