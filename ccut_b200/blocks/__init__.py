"""Drop-ins for the reference's ``ccut.blocks`` functions on the MoE path."""
