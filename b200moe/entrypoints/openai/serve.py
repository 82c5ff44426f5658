"""Console entry point ``b200moe-server`` (reference console script: s4000-server)."""
from b200moe.entrypoints.openai.api_server import main

if __name__ == "__main__":
    main()
