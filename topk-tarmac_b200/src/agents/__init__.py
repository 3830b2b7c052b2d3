"""Drop-in communication module with the reference's names and signatures."""
