"""Experiments plane: prototypes that sit beside the serving stack (PHO index, training/chat engine)."""
