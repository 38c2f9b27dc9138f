"""Minimal stand-in for the comfy_kitchen surface tilegen's backend calls.

Only what tilegen/comfyui/backend.py touches: the backend registry, the
constraint objects, the eager int8_linear and the input activations.  The
eager int8_linear here is a plain torch implementation of int8 ConvRot, enough
to check that the tilegen backend delegates to it unchanged.
"""
