"""``nangila_ddp/examples/minigpt_train.py`` entry point: random-token toy
DDP training with the compression hook."""
from mini_nangila_b200.apps.minigpt_train import main

if __name__ == "__main__":
    main()
