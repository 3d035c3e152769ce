"""Drop-in modules named after the reference's ``vflash.native`` modules they replace."""
