#:set architecture = [('Reshape', ('W', 3), ['output0'], [[6, 4]], [1]), ('MatMul', ['x', 'output0'], [2]), ('Add', ['x'], [[1, 1, 1, 4], [], 2]), ('Relu', ['x'], [2]), ('Add', ['x'], [[1, 1, 1, 4], [], 2]), ('Tanh', ['x'], [2])]
#:set inputs = [['output0', 2]]
#:set trueInputs = [['x', [1, 6]]]
#:set outShape = [['y', [1, 4]]]
#:set outputs = {'y': 'x'}
