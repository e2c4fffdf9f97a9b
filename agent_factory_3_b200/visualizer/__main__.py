"""python -m agent_factory_3_b200.visualizer batch_0001.json -o batch_0001.html"""
from .app import main

main()
