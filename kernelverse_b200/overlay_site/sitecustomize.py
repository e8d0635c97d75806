# Activates the kernelverse_b200 operator-registry overlay in every interpreter that has
# this directory on PYTHONPATH (KernelVerse evaluates cases in spawned subprocesses).
try:
    from kernelverse_b200.registry_overlay import install_import_hook

    install_import_hook()
except Exception:  # the overlay is optional: never break interpreter start-up
    pass
