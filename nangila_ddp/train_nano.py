"""``nangila_ddp/train_nano.py`` entry point (same flags), run by torchrun:
TinyGPT DDP training with the compression hook."""
from mini_nangila_b200.apps.train_nano import main

if __name__ == "__main__":
    main()
