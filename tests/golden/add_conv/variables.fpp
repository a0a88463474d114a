#:set architecture = [('Conv', ['x'], [[1, 1], [3, 3], [1, 1, 1, 1], [1, 1]]), ('Add', ['x'], [[1, 3, 6, 6], [3, 6, 4, 6], 4]), ('Relu', ['x'], [4]), ('MaxPool', ['x'], [0, [0, 0, 0, 0], [2, 2]]), ('Add', ['x'], [[1, 3, 3, 3], [3, 3, 4, 3], 4]), ('Sigmoid', ['x'], [4]), ('Reshape', ('x', 4), ['output0'], [[1, 27]], [0])]
#:set inputs = [['output0', 2]]
#:set trueInputs = [['x', [1, 2, 6, 6]]]
#:set outShape = [['y', [1, 27]]]
#:set outputs = {'y': 'output0'}
