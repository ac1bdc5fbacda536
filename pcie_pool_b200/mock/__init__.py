"""mock"""
