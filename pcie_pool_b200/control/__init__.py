"""control"""
