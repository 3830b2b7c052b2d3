"""Drop-in kernel modules with the reference's names and signatures."""
